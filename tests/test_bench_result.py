"""The bench-result file (bench_result.rs:1-122): schema, field order,
serde_json number text, pretty layout and the SHA-256 fingerprint.  No GPU."""
import hashlib
import json

from rustane_b200 import bench_result as br
from rustane_b200.sweep import SWEEP, sweep_config, sweep_tokens


def sample():
    return br.BenchResult(
        schema_version=1, rustane_version="0.1.0", git_sha="abc1234", benchmark="sweep_600m_a",
        config=br.ModelInfo(name="600m-A", dim=1536, hidden=4096, heads=12, nlayers=20, seq=512,
                            params_m=578.876928),
        results=br.TimingResults(ms_per_step=961.0, ms_fwd=235.25, ms_bwd=644.0, ms_upd=58.5, tok_per_s=533.0,
                                 loss_start=9.0108, loss_end=8.986, loss_delta=-0.0248),
        loss_trace=[9.0108, 9.0, 8.986],
        hardware=br.HardwareInfo(chip="NVIDIA B200", cores_perf=224, cores_eff=0, ram_gb=2015,
                                 macos="Ubuntu 24.04", kernel="6.8.0"),
        timestamp_utc="2026-03-18T18:30:00Z")


COMPACT = ('{"schema_version":1,"rustane_version":"0.1.0","git_sha":"abc1234","benchmark":"sweep_600m_a",'
           '"config":{"name":"600m-A","dim":1536,"hidden":4096,"heads":12,"nlayers":20,"seq":512,'
           '"params_m":578.876928},'
           '"results":{"ms_per_step":961.0,"ms_fwd":235.25,"ms_bwd":644.0,"ms_upd":58.5,"tok_per_s":533.0,'
           '"loss_start":9.0108,"loss_end":8.986,"loss_delta":-0.0248},'
           '"loss_trace":[9.0108,9.0,8.986],'
           '"hardware":{"chip":"NVIDIA B200","cores_perf":224,"cores_eff":0,"ram_gb":2015,'
           '"macos":"Ubuntu 24.04","kernel":"6.8.0"},'
           '"submitter":{"name":"","x_handle":""},"timestamp_utc":"2026-03-18T18:30:00Z","fingerprint":""}')


def test_compact_json_is_serde_layout():
    assert br.to_json(sample()) == COMPACT


def test_fingerprint_is_sha256_of_compact_json_without_fingerprint():
    r = sample()
    r.fingerprint = br.compute_fingerprint(r)
    assert r.fingerprint == hashlib.sha256(COMPACT.encode()).hexdigest()
    assert br.compute_fingerprint(r) == r.fingerprint  # independent of the stored value


def test_pretty_json_round_trips(tmp_path):
    r = sample()
    text = br.to_json(r, pretty=True)
    assert text.startswith('{\n  "schema_version": 1,\n  "rustane_version": "0.1.0",')
    assert '\n  "loss_trace": [\n    9.0108,\n    9.0,\n    8.986\n  ],\n' in text
    assert json.loads(text) == json.loads(COMPACT)
    p = br.write_result(r, tmp_path / "target" / "bench-result.json", out=lambda s: None)
    assert json.loads(p.read_text())["results"]["tok_per_s"] == 533.0


def test_f32_fields_print_f32_digits_and_strings_escape():
    r = sample()
    r.results.ms_fwd = 0.1 + 0.2  # as f32: 0.3
    r.loss_trace = [float("nan"), 1e-7]
    r.submitter = br.Submitter(name='a"b\\c\n', x_handle="")
    s = br.to_json(r)
    assert '"ms_fwd":0.3,' in s and '"loss_trace":[null,1e-7]' in s
    assert '"name":"a\\"b\\\\c\\n"' in s
    r.loss_trace = []
    assert '"loss_trace": [],' in br.to_json(r, pretty=True)


def test_sweep_table_and_tokens():
    assert len(SWEEP) == 27
    cfg = sweep_config("600m-B")  # bench_param_sweep.rs custom_config(1280, 3456, 10, 28, 512)
    assert (cfg.dim, cfg.hidden, cfg.heads, cfg.nlayers, cfg.seq, cfg.hd, cfg.vocab) == \
        (1280, 3456, 10, 28, 512, 128, 8192)
    tok, tgt = sweep_tokens(sweep_config("600m-E"), 2)
    assert tok.size == 512 and list(tok[:3]) == [7, 38, 69] and list(tgt[:2]) == [38, 69]
    assert tok[256] == 7 and tgt[255] == (256 * 31 + 7) % 8192
