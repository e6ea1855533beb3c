"""Benchmark result file (crates/engine/src/bench_result.rs:1-122): the same
schema, field order and JSON number text as the reference's
`target/bench-result.json`, so B200 runs can be compared and submitted the
same way.

The struct fields and their Rust types are kept (f32 fields print with f32
shortest digits, as serde_json does).  HardwareInfo is filled on Linux:
`chip` is the accelerator's name (e.g. "NVIDIA B200"), `cores_perf` the host's
logical CPUs, `cores_eff` 0, `ram_gb` the host memory in GiB, `macos` the OS
release (the field name is the schema's), `kernel` the kernel release.
"""
from __future__ import annotations

import hashlib
import os
import platform
import subprocess
from dataclasses import dataclass, field, fields, replace
from pathlib import Path

from .rustfmt import json_f32, json_f64

SCHEMA_VERSION = 1
RUSTANE_VERSION = "0.1.0"  # the reference workspace version (Cargo.toml)


@dataclass
class ModelInfo:  # bench_result.rs:24-33
    name: str
    dim: int
    hidden: int
    heads: int
    nlayers: int
    seq: int
    params_m: float  # f64


@dataclass
class TimingResults:  # bench_result.rs:35-45 (all f32)
    ms_per_step: float
    ms_fwd: float
    ms_bwd: float
    ms_upd: float
    tok_per_s: float
    loss_start: float
    loss_end: float
    loss_delta: float


@dataclass
class HardwareInfo:  # bench_result.rs:47-55
    chip: str = ""
    cores_perf: int = 0
    cores_eff: int = 0
    ram_gb: int = 0
    macos: str = ""
    kernel: str = ""


@dataclass
class Submitter:  # bench_result.rs:57-61
    name: str = ""
    x_handle: str = ""


@dataclass
class BenchResult:  # bench_result.rs:9-22
    schema_version: int
    rustane_version: str
    git_sha: str
    benchmark: str
    config: ModelInfo
    results: TimingResults
    loss_trace: list  # Vec<f32>
    hardware: HardwareInfo
    submitter: Submitter = field(default_factory=Submitter)
    timestamp_utc: str = ""
    fingerprint: str = ""


# fields serialised as f32 / f64 (everything else is an int, a string, a list or a struct)
_F32 = {"ms_per_step", "ms_fwd", "ms_bwd", "ms_upd", "tok_per_s", "loss_start", "loss_end", "loss_delta",
        "loss_trace"}
_F64 = {"params_m"}


def _str(s: str) -> str:
    out = ['"']
    for ch in s:
        o = ord(ch)
        if ch == '"':
            out.append('\\"')
        elif ch == "\\":
            out.append("\\\\")
        elif ch in "\b\f\n\r\t":
            out.append({"\b": "\\b", "\f": "\\f", "\n": "\\n", "\r": "\\r", "\t": "\\t"}[ch])
        elif o < 0x20:
            out.append(f"\\u{o:04x}")
        else:
            out.append(ch)
    out.append('"')
    return "".join(out)


def _value(v, name: str, indent: int | None, depth: int) -> str:
    if hasattr(v, "__dataclass_fields__"):
        return _object([(f.name, getattr(v, f.name)) for f in fields(v)], indent, depth)
    if isinstance(v, str):
        return _str(v)
    if isinstance(v, (list, tuple)):
        items = [_value(x, name, indent, depth + 1) for x in v]
        if not items:
            return "[]"
        if indent is None:
            return "[" + ",".join(items) + "]"
        pad, pad_in = " " * (indent * depth), " " * (indent * (depth + 1))
        return "[\n" + ",\n".join(pad_in + x for x in items) + "\n" + pad + "]"
    if name in _F32:
        return json_f32(v)
    if name in _F64:
        return json_f64(v)
    return str(int(v))


def _object(items, indent: int | None, depth: int) -> str:
    if not items:
        return "{}"
    if indent is None:
        return "{" + ",".join(f"{_str(k)}:{_value(v, k, None, depth + 1)}" for k, v in items) + "}"
    pad, pad_in = " " * (indent * depth), " " * (indent * (depth + 1))
    body = ",\n".join(f"{pad_in}{_str(k)}: {_value(v, k, indent, depth + 1)}" for k, v in items)
    return "{\n" + body + "\n" + pad + "}"


def to_json(result: BenchResult, pretty: bool = False) -> str:
    """serde_json::to_string (compact) / to_string_pretty (2-space indent)."""
    return _value(result, "", 2 if pretty else None, 0)


def compute_fingerprint(result: BenchResult) -> str:
    """SHA-256 hex of the compact JSON with an empty fingerprint (bench_result.rs:85-93)."""
    return hashlib.sha256(to_json(replace(result, fingerprint="")).encode()).hexdigest()


def _run(cmd: list[str]) -> str:
    try:
        return subprocess.run(cmd, capture_output=True, text=True, timeout=10).stdout.strip()
    except (OSError, subprocess.SubprocessError):
        return ""


def git_sha() -> str:
    """bench_result.rs:75-78 (empty outside a git checkout)."""
    return _run(["git", "-C", str(Path(__file__).resolve().parent), "rev-parse", "--short", "HEAD"])


def utc_timestamp() -> str:
    """bench_result.rs:80-83."""
    import datetime
    return datetime.datetime.now(datetime.timezone.utc).strftime("%Y-%m-%dT%H:%M:%SZ")


def collect_hardware_info(chip: str | None = None) -> HardwareInfo:
    """HardwareInfo of this host (bench_result.rs:63-73 reads sysctl on macOS)."""
    if chip is None:
        chip = _run(["nvidia-smi", "--query-gpu=name", "--format=csv,noheader"]).splitlines()[:1]
        chip = chip[0].strip() if chip else platform.processor()
    ram = 0
    try:
        with open("/proc/meminfo") as f:
            for line in f:
                if line.startswith("MemTotal:"):
                    ram = int(line.split()[1]) * 1024 // (1 << 30)
                    break
    except OSError:
        pass
    os_release = ""
    try:
        with open("/etc/os-release") as f:
            for line in f:
                if line.startswith("PRETTY_NAME="):
                    os_release = line.split("=", 1)[1].strip().strip('"')
    except OSError:
        pass
    return HardwareInfo(chip=chip, cores_perf=os.cpu_count() or 0, cores_eff=0, ram_gb=ram, macos=os_release,
                        kernel=platform.release())


def write_result(result: BenchResult, path="target/bench-result.json", out=print) -> Path:
    """bench_result.rs:95-102: pretty JSON to `path` (directories created)."""
    p = Path(path)
    p.parent.mkdir(parents=True, exist_ok=True)
    p.write_text(to_json(result, pretty=True))
    out(f"\n  Result saved to {p}")
    return p
