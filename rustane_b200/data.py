"""Training data, val bits-per-byte and checkpoints: the host side of the
reference's training loop over librustane_cuda.so's host I/O entry points.

    TokenData.open(path)        data.rs:11-39   (mmap'd little-endian u16 tokens)
    TokenBytes.load(path)       data.rs:41-64   (int32 byte length per token id)
    compute_bpb(...)            data.rs:66-89
    random_position(...)        data.rs:91-95   (the training loop's LCG positions)
    save_checkpoint(...)        bin/train.rs:165-202 (RSTK version 1; version 2 adds AdamW moments)
    load_checkpoint(...)        reader for both versions (the reference has none)

Every call goes through the C ABI (rt_tokens_*, rt_compute_bpb, rt_checkpoint_*);
errors raise RustaneError where the reference panics.
"""
from __future__ import annotations

import ctypes
from pathlib import Path

import numpy as np

from ._lib import RustaneError, lib
from .model import ModelConfig
from .tensors import ModelOptState, ModelTensors


def _u32p(a: np.ndarray):
    return a.ctypes.data_as(ctypes.POINTER(ctypes.c_uint32))


def _check(rc: int, what: str) -> None:
    if rc != 0:
        raise RustaneError(rc, what)


class TokenData:
    """Memory-mapped token file (TokenData, data.rs:11-39)."""

    def __init__(self, handle: ctypes.c_void_p, path: Path):
        self._h = handle
        self.path = path
        n = ctypes.c_int64()
        _check(lib().rt_tokens_len(self._h, ctypes.byref(n)), str(path))
        self._n = n.value

    @classmethod
    def open(cls, path) -> "TokenData":
        h = ctypes.c_void_p()
        _check(lib().rt_tokens_open(str(path).encode(), ctypes.byref(h)), f"open {path}")
        return cls(h, Path(path))

    def close(self) -> None:
        if self._h is not None and self._h.value:
            lib().rt_tokens_close(self._h)
        self._h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __len__(self) -> int:
        return self._n

    def len(self) -> int:
        return self._n

    def tokens(self, start: int, length: int) -> np.ndarray:
        """Tokens [start, start + length) as uint32 (data.rs:35-38)."""
        out = np.empty(length, np.uint32)
        _check(lib().rt_tokens_read(self._h, start, length, _u32p(out)), f"tokens({start}, {length})")
        return out

    def token(self, pos: int) -> int:
        return int(self.tokens(pos, 1)[0])

    def train_window(self, step: int, micro: int, seq: int) -> tuple[np.ndarray, np.ndarray]:
        """(input, target) of microbatch `micro` at `step` (bin/train.rs:285-290)."""
        tok, tgt = np.empty(seq, np.uint32), np.empty(seq, np.uint32)
        _check(lib().rt_tokens_train_window(self._h, step, micro, seq, _u32p(tok), _u32p(tgt)), "train window")
        return tok, tgt

    def val_window(self, vs: int, seq: int) -> tuple[np.ndarray, np.ndarray]:
        """(input, target) of validation step `vs` (bin/train.rs:128-131)."""
        tok, tgt = np.empty(seq, np.uint32), np.empty(seq, np.uint32)
        _check(lib().rt_tokens_val_window(self._h, vs, seq, _u32p(tok), _u32p(tgt)), "val window")
        return tok, tgt


class TokenBytes:
    """Byte length of each token id, 0 for special tokens (TokenBytes, data.rs:41-64)."""

    def __init__(self, table: np.ndarray):
        self.bytes = np.ascontiguousarray(table, dtype=np.int32)

    @classmethod
    def load(cls, path) -> "TokenBytes":
        raw = Path(path).read_bytes()
        return cls(np.frombuffer(raw[: len(raw) // 4 * 4], dtype="<i4").astype(np.int32))

    def byte_len(self, token_id: int) -> int:
        return int(self.bytes[token_id])


def compute_bpb(losses, targets, token_bytes: TokenBytes) -> tuple[float, float, int]:
    """(bpb, total_nats, total_bytes) over per-token losses (data.rs:66-89)."""
    losses = np.ascontiguousarray(losses, dtype=np.float32)
    targets = np.ascontiguousarray(targets, dtype=np.uint32)
    if losses.size != targets.size:
        raise ValueError("losses and targets differ in length")
    bpb, nats, nbytes = ctypes.c_float(), ctypes.c_float(), ctypes.c_int64()
    _check(lib().rt_compute_bpb(losses.ctypes.data_as(ctypes.POINTER(ctypes.c_float)), _u32p(targets), losses.size,
                                token_bytes.bytes.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)),
                                token_bytes.bytes.size, ctypes.byref(bpb), ctypes.byref(nats), ctypes.byref(nbytes)),
           "compute_bpb")
    return bpb.value, nats.value, nbytes.value


def random_position(step: int, micro: int, max_pos: int) -> int:
    """data.rs:91-95 (u64 wrapping arithmetic)."""
    m = (1 << 64) - 1
    return ((step * 7919 & m) + (micro * 104729 & m) & m) % max_pos


def checkpoint_path(dir_, step: int) -> Path:
    """ckpt_{step:06}.bin inside `dir_` (bin/train.rs:173)."""
    return Path(dir_) / f"ckpt_{step:06d}.bin"


def save_checkpoint(cfg: ModelConfig, weights: ModelTensors, opt: ModelOptState | None, step: int, dir_,
                    with_opt: bool = False) -> Path:
    """save_checkpoint (bin/train.rs:165-202): writes dir/ckpt_{step:06}.bin.
    Version 1 (the reference's format) unless `with_opt`, which writes version
    2 with the AdamW moments appended."""
    Path(dir_).mkdir(parents=True, exist_ok=True)
    path = checkpoint_path(dir_, step)
    c_cfg = cfg.to_c()
    w = weights.c_ptrs()
    m = v = None
    if with_opt:
        if opt is None:
            raise ValueError("with_opt needs the optimizer state")
        m, v = opt.m.c_ptrs(), opt.v.c_ptrs()
    _check(lib().rt_checkpoint_write(str(path).encode(), ctypes.byref(c_cfg), step, ctypes.byref(w),
                                     ctypes.byref(m) if m is not None else None,
                                     ctypes.byref(v) if v is not None else None), f"write {path}")
    return path


def load_checkpoint(path, cfg: ModelConfig, with_opt: bool = True) -> tuple[ModelTensors, ModelOptState | None, int,
                                                                            int]:
    """Read an RSTK checkpoint written for `cfg`: (weights, opt or None, step,
    version).  `opt` is filled when the file is version 2 and `with_opt`."""
    c_cfg = cfg.to_c()
    weights = ModelTensors.zeros(cfg)
    opt = ModelOptState.zeros(cfg) if with_opt else None
    w = weights.c_ptrs()
    m, v = (opt.m.c_ptrs(), opt.v.c_ptrs()) if opt is not None else (None, None)
    step, version = ctypes.c_uint32(), ctypes.c_uint32()
    _check(lib().rt_checkpoint_read(str(path).encode(), ctypes.byref(c_cfg), ctypes.byref(step),
                                    ctypes.byref(version), ctypes.byref(w),
                                    ctypes.byref(m) if m is not None else None,
                                    ctypes.byref(v) if v is not None else None), f"read {path}")
    if version.value != 2:
        opt = None
    return weights, opt, step.value, version.value
