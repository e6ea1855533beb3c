"""C-ABI checks that need no GPU: librustane_cuda.so loads, exports every
function include/rustane_cuda.h declares, the ctypes binding covers them all,
and the host-only helpers agree with the oracle (no device compute here)."""
import re

import numpy as np

import pyoracle as po
from rustane_b200 import _lib, engine
from rustane_b200.model import ModelConfig


def declared_functions() -> list[str]:
    text = _lib.HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return re.findall(r"RT_API\s+[\w\s\*]+?\b(rt_\w+)\s*\(", text)


def test_header_declares_entry_points():
    names = declared_functions()
    assert len(names) >= 30
    assert len(names) == len(set(names))


def test_library_exports_every_declared_symbol():
    L = _lib.lib()
    missing = [n for n in declared_functions() if not hasattr(L, n)]
    assert not missing, missing


def test_binding_covers_every_declared_symbol():
    assert set(declared_functions()) == set(_lib.SIGNATURES)


def test_lcg_fill_matches_oracle_bitwise():  # layer.rs:404-413
    for n, scale in [(7, 1.0), (1536 * 1536, 1 / np.sqrt(np.float32(1536))), (8192 * 64, 0.005)]:
        a = engine.lcg_random_vec(n, float(scale))
        b = po.random_vec(n, float(scale))
        assert np.array_equal(a, b)


def test_random_weights_match_oracle_reference_init():
    cfg = ModelConfig.custom(256, 512, 2, 2, seq=128, vocab=512)
    a, b = engine.random_weights(cfg), po.reference_init(cfg)
    for (na, x), (_, y) in zip(a.tensors(), b.tensors()):
        assert np.array_equal(x, y), na


def test_learning_rate_matches_oracle():
    tc = engine.TrainConfig()
    otc = po.default_train_config()
    for step in (0, 1, 50, 99, 100, 101, 5000, 9999):
        assert engine.learning_rate(step, tc) == po.learning_rate(step, otc)


def test_train_positions_match_oracle():
    import ctypes
    out = (ctypes.c_int64 * 10)()
    po.lib().or_train_positions(17, 10, 1_000_000, 512, out)
    assert engine.train_positions(17, 10, 1_000_000, 512) == list(out)


def test_rt_last_error_without_context_is_safe():
    assert isinstance(_lib.lib().rt_last_error(None), bytes)
