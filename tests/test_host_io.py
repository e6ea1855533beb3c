"""Host I/O of the training loop, through the C ABI (no GPU): the u16 token
files and sampling windows (data.rs:11-39, 91-95; bin/train.rs:128-131,
285-290), compute_bpb (data.rs:66-89) and the RSTK checkpoint
(bin/train.rs:165-202), each against an independent numpy restatement."""
import struct

import numpy as np
import pytest

from rustane_b200 import RustaneError
from rustane_b200.data import (TokenBytes, TokenData, checkpoint_path, compute_bpb, load_checkpoint,
                               random_position, save_checkpoint)
from rustane_b200.model import ModelConfig
from rustane_b200.tensors import LAYER_FIELDS, ModelOptState, ModelTensors

SMALL = ModelConfig.custom(64, 96, 1, 2, seq=16, vocab=50, hd=64)


def write_tokens(path, arr):
    path.write_bytes(np.asarray(arr, dtype="<u2").tobytes())


@pytest.fixture
def token_file(tmp_path):
    rng = np.random.default_rng(7)
    arr = rng.integers(0, 65536, size=10007, dtype=np.uint32)
    arr[:4] = [0, 1, 255, 65535]  # byte-order edge values
    p = tmp_path / "train.bin"
    write_tokens(p, arr)
    return p, arr


def test_token_data_reads_le_u16(token_file):
    p, arr = token_file
    with TokenData.open(p) as td:
        assert len(td) == arr.size
        assert np.array_equal(td.tokens(0, arr.size), arr)
        assert td.token(3) == 65535
        assert np.array_equal(td.tokens(500, 0), np.empty(0, np.uint32))
        with pytest.raises(RustaneError):
            td.tokens(arr.size - 3, 4)
        with pytest.raises(RustaneError):
            td.tokens(-1, 2)


def test_odd_file_length_drops_last_byte(tmp_path):
    p = tmp_path / "odd.bin"
    p.write_bytes(bytes([1, 0, 2, 0, 9]))
    with TokenData.open(p) as td:  # data.rs:22 n_tokens = len / 2
        assert len(td) == 2 and list(td.tokens(0, 2)) == [1, 2]


def test_open_missing_file_raises(tmp_path):
    with pytest.raises(RustaneError):
        TokenData.open(tmp_path / "nope.bin")


@pytest.mark.parametrize("seq", [16, 512])
def test_train_windows_follow_reference_lcg(token_file, seq):
    p, arr = token_file
    max_pos = arr.size - seq - 1
    with TokenData.open(p) as td:
        for step in [0, 1, 7, 1234, 71999, 2**32 - 1]:
            for micro in [0, 1, 9, 2**32 - 1]:
                pos = (step * 7919 + micro * 104729) % max_pos  # bin/train.rs:285
                assert pos == random_position(step, micro, max_pos)
                tok, tgt = td.train_window(step, micro, seq)
                assert np.array_equal(tok, arr[pos:pos + seq])
                assert np.array_equal(tgt, arr[pos + 1:pos + seq + 1])


def test_val_windows_follow_reference(token_file):
    p, arr = token_file
    seq = 512
    max_pos = arr.size - seq - 1
    with TokenData.open(p) as td:
        for vs in [0, 1, 19, 20, 1000]:
            pos = (vs * seq) % max_pos  # bin/train.rs:129
            tok, tgt = td.val_window(vs, seq)
            assert np.array_equal(tok, arr[pos:pos + seq])
            assert np.array_equal(tgt, arr[pos + 1:pos + seq + 1])


def test_window_needs_seq_plus_two_tokens(tmp_path):
    p = tmp_path / "short.bin"
    write_tokens(p, np.arange(17))
    with TokenData.open(p) as td:
        with pytest.raises(RustaneError):  # max_pos = 17 - 16 - 1 = 0: the reference divides by zero
            td.train_window(0, 0, 16)
        tok, tgt = td.train_window(5, 3, 15)  # max_pos = 1: every window starts at 0
        assert list(tok) == list(range(15)) and list(tgt) == list(range(1, 16))


def bpb_restated(losses, targets, table):
    nats = np.float32(0)
    nbytes = 0
    for loss, t in zip(losses, targets):
        bl = int(table[t])
        if bl > 0:
            nats = np.float32(nats + np.float32(loss))
            nbytes += bl
    bpb = np.float32(nats / (np.float32(np.log(2)) * np.float32(nbytes))) if nbytes else np.float32(0)
    return float(bpb), float(nats), nbytes


def test_compute_bpb_matches_restatement(tmp_path):
    rng = np.random.default_rng(3)
    table = rng.integers(1, 9, size=8192).astype(np.int32)
    table[rng.integers(0, 8192, size=300)] = 0  # special tokens count no bytes
    (tmp_path / "token_bytes.bin").write_bytes(table.astype("<i4").tobytes())
    tb = TokenBytes.load(tmp_path / "token_bytes.bin")
    assert np.array_equal(tb.bytes, table) and tb.byte_len(5) == table[5]
    losses = rng.uniform(0.0, 12.0, size=20 * 512).astype(np.float32)
    targets = rng.integers(0, 8192, size=losses.size).astype(np.uint32)
    targets[:50] = np.flatnonzero(table == 0)[:50]
    got = compute_bpb(losses, targets, tb)
    assert got == bpb_restated(losses, targets, table)


def test_compute_bpb_edge_cases():
    tb = TokenBytes(np.array([0, 3, 1], np.int32))
    assert compute_bpb(np.zeros(0, np.float32), np.zeros(0, np.uint32), tb) == (0.0, 0.0, 0)
    assert compute_bpb(np.array([2.0], np.float32), np.array([0], np.uint32), tb) == (0.0, 0.0, 0)
    bpb, nats, nb = compute_bpb(np.array([1.0, 2.0], np.float32), np.array([1, 2], np.uint32), tb)
    assert (nats, nb) == (3.0, 4) and bpb == pytest.approx(3.0 / (np.log(2) * 4), rel=1e-6)
    with pytest.raises(RustaneError):  # id past the table (the reference panics on the index)
        compute_bpb(np.array([1.0], np.float32), np.array([3], np.uint32), tb)


def filled(cfg, seed):
    t = ModelTensors.normal(cfg, seed=seed, std=0.5)
    for L in t.layers:
        L.gamma1[...] = np.float32(seed)
    return t


def reference_v1_bytes(cfg, w, step):
    """bin/train.rs:175-193, restated: header then fp32 LE tensors in order."""
    out = b"RSTK" + struct.pack("<6I", 1, step, cfg.dim, cfg.nlayers, cfg.vocab, cfg.seq)
    out += w.embed.astype("<f4").tobytes() + w.gamma_final.astype("<f4").tobytes()
    for L in w.layers:
        for f in LAYER_FIELDS:
            out += getattr(L, f).astype("<f4").tobytes()
    return out


def test_checkpoint_v1_is_reference_format(tmp_path):
    w = filled(SMALL, 1)
    path = save_checkpoint(SMALL, w, None, 42, tmp_path / "ck")
    assert path == checkpoint_path(tmp_path / "ck", 42) and path.name == "ckpt_000042.bin"
    assert path.read_bytes() == reference_v1_bytes(SMALL, w, 42)
    w2, opt, step, version = load_checkpoint(path, SMALL)
    assert (step, version, opt) == (42, 1, None)
    for (_, a), (_, b) in zip(w.tensors(), w2.tensors()):
        assert np.array_equal(a, b)


def test_checkpoint_v2_roundtrips_optimizer_state(tmp_path):
    w = filled(SMALL, 2)
    opt = ModelOptState(filled(SMALL, 3), filled(SMALL, 4))
    path = save_checkpoint(SMALL, w, opt, 7, tmp_path, with_opt=True)
    raw = path.read_bytes()
    v1 = reference_v1_bytes(SMALL, w, 7)
    assert raw[4:8] == struct.pack("<I", 2) and raw[8:len(v1)] == v1[8:]
    assert len(raw) == len(v1) + 2 * (len(v1) - 28)
    w2, opt2, step, version = load_checkpoint(path, SMALL)
    assert (step, version) == (7, 2)
    for a_, b_ in [(w, w2), (opt.m, opt2.m), (opt.v, opt2.v)]:
        for (_, a), (_, b) in zip(a_.tensors(), b_.tensors()):
            assert np.array_equal(a, b)
    w3, opt3, _, _ = load_checkpoint(path, SMALL, with_opt=False)
    assert opt3 is None and np.array_equal(w3.embed, w.embed)


def test_checkpoint_reader_rejects_bad_files(tmp_path):
    path = save_checkpoint(SMALL, filled(SMALL, 1), None, 1, tmp_path)
    for other in [SMALL.with_(dim=128), SMALL.with_(nlayers=3), SMALL.with_(vocab=51), SMALL.with_(seq=32)]:
        with pytest.raises(RustaneError):
            load_checkpoint(path, other)
    raw = path.read_bytes()
    (tmp_path / "trunc.bin").write_bytes(raw[:-4])
    (tmp_path / "magic.bin").write_bytes(b"RSTX" + raw[4:])
    (tmp_path / "ver.bin").write_bytes(raw[:4] + struct.pack("<I", 3) + raw[8:])
    for name in ["trunc.bin", "magic.bin", "ver.bin", "missing.bin"]:
        with pytest.raises(RustaneError):
            load_checkpoint(tmp_path / name, SMALL)
    with pytest.raises(ValueError):
        save_checkpoint(SMALL, filled(SMALL, 1), None, 1, tmp_path, with_opt=True)
