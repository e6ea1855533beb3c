"""Number formatting of the reference's Rust output, so logs and JSON files
read byte for byte like the reference's.

- `display_f32`: Rust `{}` of an f32 (shortest round-trip digits, never an
  exponent: 1e-8 prints as 0.00000001, 256.0 as 256).
- `exp_f32`: Rust `{:.Ne}` (3e-4 at .2 prints 3.00e-4: no '+', no exponent padding).
- `json_f32` / `json_f64`: serde_json's number text (ryu shortest digits, laid
  out as 961.0, 0.001, 1e-7, 1.5e30; NaN and infinities as null).
"""
from __future__ import annotations

import math

import numpy as np


def display_f32(x) -> str:
    x = np.float32(x)
    if not np.isfinite(x):
        return "NaN" if np.isnan(x) else ("inf" if x > 0 else "-inf")
    return np.format_float_positional(x, unique=True, trim="-")


def exp_f32(x, prec: int) -> str:
    x = float(np.float32(x))
    if not math.isfinite(x):
        return "NaN" if math.isnan(x) else ("inf" if x > 0 else "-inf")
    mant, exp = f"{x:.{prec}e}".split("e")
    return f"{mant}e{int(exp)}"


def _shortest_digits(x: float, f32: bool) -> tuple[str, int]:
    """(digits, decimal exponent of the last digit) of the shortest round-trip form of x > 0."""
    v = np.float32(x) if f32 else np.float64(x)
    mant, exp = np.format_float_scientific(v, unique=True, trim="-").split("e")
    digits = mant.replace(".", "").rstrip("0") or "0"
    return digits, int(exp) - (len(digits) - 1)


# ryu's layout limits: plain digits up to 10^13 (f32) / 10^16 (f64), leading
# zeros after the point down to 10^-6 (f32) / 10^-5 (f64).
def _ryu_layout(x: float, f32: bool) -> str:
    if math.isnan(x) or math.isinf(x):
        return "null"
    if x == 0:
        return "-0.0" if math.copysign(1.0, x) < 0 else "0.0"
    hi, lo = (13, -6) if f32 else (16, -5)
    sign = "-" if x < 0 else ""
    digits, k = _shortest_digits(abs(x), f32)
    n = len(digits)
    kk = n + k  # 10^(kk-1) <= |x| < 10^kk
    if 0 <= k and kk <= hi:
        body = digits + "0" * k + ".0"
    elif 0 < kk <= hi:
        body = digits[:kk] + "." + digits[kk:]
    elif lo < kk <= 0:
        body = "0." + "0" * (-kk) + digits
    elif n == 1:
        body = f"{digits}e{kk - 1}"
    else:
        body = f"{digits[0]}.{digits[1:]}e{kk - 1}"
    return sign + body


def json_f32(x) -> str:
    return _ryu_layout(float(np.float32(x)), True)


def json_f64(x) -> str:
    return _ryu_layout(float(x), False)
