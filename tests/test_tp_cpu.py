"""Tensor-parallel forward on CPU ranks (gloo, world size 2).

The library's tensor-parallel forward (forward-only contexts joined with
RT_DIST_TENSOR_PARALLEL) shards each layer over the ranks by the partition
rt_tp_shard returns: Wq / Wk / Wv are column shards by heads, Wo the matching
row shard, W1 / W3 column shards and W2 the matching row shard by 64-column
hidden units.  Each rank computes its heads' attention and its hidden units'
SwiGLU, and the two row-parallel products (after Wo, after W2) are summed
over the ranks by an all-reduce before the residual add.  Embedding, final
RMSNorm, tied logits and loss are replicated.

Here two gloo ranks run that protocol with the oracle's own layer math
(layer.rs:443-548 restated in oracle/oracle.cpp) on a configuration whose
split is uneven in both dimensions (3 heads -> 2 + 1, 5 hidden units ->
3 + 2), and the result must equal the unsharded oracle forward
(full_model.rs:187-247): final hidden state, logits and loss.

Each row-parallel product is obtained from the oracle's layer forward with
the other half of the layer switched off: with W1 = W3 = W2 = 0 the layer
returns x + alpha * (attn Wo) exactly, and with Wo = 0 it returns
x2 + alpha * (gate W2^T) with x2 = x; subtracting the input leaves the rank's
partial, which is what the GPU all-reduces.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

CFG_ARGS = dict(dim=384, hidden=320, heads=3, nlayers=2, seq=32, vocab=96)
TOL = 1e-4  # fp32 on both sides; only the summation order differs


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _cfg():
    from rustane_b200.model import ModelConfig
    return ModelConfig.custom(CFG_ARGS["dim"], CFG_ARGS["hidden"], CFG_ARGS["heads"], CFG_ARGS["nlayers"],
                              seq=CFG_ARGS["seq"], vocab=CFG_ARGS["vocab"])


def _data(cfg):
    rng = np.random.default_rng(91)
    tok = rng.integers(0, cfg.vocab, cfg.seq).astype(np.uint32)
    tgt = rng.integers(0, cfg.vocab, cfg.seq).astype(np.uint32)
    return tok, tgt


def _local_layers(cfg, L, head0, heads_loc, hid0, hid_loc):
    """This rank's (attention-half, FFN-half) layer tensors for the oracle."""
    from rustane_b200.tensors import LayerTensors
    hd = cfg.hd
    q = slice(head0 * hd, (head0 + heads_loc) * hd)
    h = slice(hid0, hid0 + hid_loc)
    cols = lambda a, s: np.ascontiguousarray(a[:, s])  # noqa: E731
    wq, wk, wv = cols(L.wq, q), cols(L.wk, q), cols(L.wv, q)
    wo = np.ascontiguousarray(L.wo[q, :])
    zeros_h = np.zeros((cfg.dim, hid_loc), np.float32)
    attn = LayerTensors(wq, wk, wv, wo, zeros_h, zeros_h.copy(), zeros_h.copy(), L.gamma1.copy(), L.gamma2.copy())
    ffn = LayerTensors(wq, wk, wv, np.zeros_like(wo), cols(L.w1, h), cols(L.w3, h), cols(L.w2, h), L.gamma1.copy(),
                       L.gamma2.copy())
    return attn, ffn


def _tail(cfg, w, x, tgt):
    """Replicated tail: final RMSNorm (cpu/rmsnorm.rs:149-183), tied logits, mean CE."""
    x = x.astype(np.float64)
    rms_inv = 1.0 / np.sqrt(np.mean(x * x, axis=0) + 1e-5)
    xn = x * rms_inv[None, :] * w.gamma_final.astype(np.float64)[:, None]
    logits = (w.embed.astype(np.float64) @ xn).T  # [S, V]
    m = logits.max(axis=1, keepdims=True)
    lse = (m[:, 0] + np.log(np.exp(logits - m).sum(axis=1)))
    loss = float(np.mean(lse - logits[np.arange(cfg.seq), tgt]))
    return logits, loss


def _worker(rank: int, world: int, port: int, out_path: str) -> None:
    import sys
    from pathlib import Path
    root = Path(__file__).resolve().parent.parent
    sys.path[:0] = [str(root), str(root / "oracle")]
    import pyoracle as po
    from rustane_b200.engine import tp_shard
    from rustane_b200.model import ModelConfig
    from rustane_b200.tensors import ModelTensors

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        cfg = _cfg()
        po.lib(threads=1)
        w = ModelTensors.normal(cfg, seed=5, std=0.05)
        tok, tgt = _data(cfg)
        head0, heads_loc, hid0, hid_loc = tp_shard(cfg.heads, cfg.hidden, world, rank)
        local = ModelConfig(dim=cfg.dim, hidden=hid_loc, heads=heads_loc, kv_heads=heads_loc, hd=cfg.hd,
                            seq=cfg.seq, nlayers=cfg.nlayers, vocab=cfg.vocab, q_dim=heads_loc * cfg.hd,
                            kv_dim=heads_loc * cfg.hd, gqa_ratio=1)
        o = po.Oracle(local, 1)
        x = np.ascontiguousarray(w.embed[tok].T)  # embedding::forward, channel-first [D, S]
        for L in w.layers:
            attn, ffn = _local_layers(cfg, L, head0, heads_loc, hid0, hid_loc)
            part = torch.from_numpy(o.layer_forward(attn, x) - x)  # alpha * attn_r Wo_r
            dist.all_reduce(part)  # the all-reduce after the row-parallel Wo product
            x2 = np.ascontiguousarray(x + part.numpy())
            part = torch.from_numpy(o.layer_forward(ffn, x2) - x2)  # alpha * gate_r W2_r^T
            dist.all_reduce(part)  # the all-reduce after the row-parallel W2 product
            x = np.ascontiguousarray(x2 + part.numpy())
        logits, loss = _tail(cfg, w, x, tgt)
        got = [None] * world
        dist.all_gather_object(got, (rank, head0, heads_loc, hid0, hid_loc, x, loss))
        if rank == 0:
            np.savez(out_path, x=x, logits=logits, loss=loss,
                     shards=np.array([g[1:5] for g in got]),
                     x_other=got[1][5], loss_other=got[1][6])
    finally:
        dist.destroy_process_group()


def test_tensor_parallel_forward_equals_single_process(tmp_path):
    import pyoracle as po
    from rustane_b200.tensors import ModelTensors

    out = str(tmp_path / "rank0.npz")
    mp.spawn(_worker, args=(2, _free_port(), out), nprocs=2, join=True)
    got = np.load(out)
    # uneven in both dimensions: 3 heads -> 2 + 1, 320 hidden columns -> 192 + 128
    assert got["shards"].tolist() == [[0, 2, 0, 192], [2, 1, 192, 128]]
    # replicated after the all-reduces: both ranks hold the same hidden state and loss
    assert np.array_equal(got["x"], got["x_other"]) and float(got["loss"]) == float(got["loss_other"])

    cfg = _cfg()
    w = ModelTensors.normal(cfg, seed=5, std=0.05)
    tok, tgt = _data(cfg)
    o = po.Oracle(cfg, 1)
    loss_ref, logits_ref, _ = o.forward(w, tok, tgt, want_logits=True)
    x_ref = np.ascontiguousarray(w.embed[tok].T)
    for L in w.layers:
        x_ref = o.layer_forward(L, x_ref)
    assert np.max(np.abs(got["x"] - x_ref)) <= TOL * np.max(np.abs(x_ref))
    assert np.max(np.abs(got["logits"] - logits_ref)) <= TOL * np.max(np.abs(logits_ref))
    assert abs(float(got["loss"]) - loss_ref) < TOL


@pytest.mark.parametrize("heads,hidden,world", [(52, 17920, 8), (32, 11008, 8), (3, 320, 2), (20, 6912, 3),
                                                (12, 4096, 1)])
def test_tp_partition_tiles_heads_and_hidden(heads, hidden, world):
    """rt_tp_shard: contiguous, non-overlapping shards covering every head and column,
    64-column hidden units, sizes differing by at most one unit."""
    from rustane_b200.engine import tp_shard
    parts = [tp_shard(heads, hidden, world, r) for r in range(world)]
    h_next = c_next = 0
    for head0, heads_loc, hid0, hid_loc in parts:
        assert head0 == h_next and hid0 == c_next
        if world > 1:
            assert hid_loc % 64 == 0
        h_next, c_next = head0 + heads_loc, hid0 + hid_loc
    assert h_next == heads and c_next == hidden
    assert max(p[1] for p in parts) - min(p[1] for p in parts) <= 1
    assert max(p[3] for p in parts) - min(p[3] for p in parts) <= (64 if world > 1 else 0)
