"""Extract the reference's published initial losses into published_losses.json.

Run in the build container, where the reference checkout is readable:
    python tests/golden/extract_published.py <reference-root>
It parses the loss0 column of the parameter-sweep tables
(results/2026-03-18_1830_param-sweep.md) and the README's 600m-A and 7B runs
(README.md:58, :70).  Those numbers come from the reference's ModelWeights::random
init and tokens (i*31+7) % vocab, so they pin the oracle's embedding, final
RMSNorm, tied logits and cross-entropy; every layer is an identity map at that
init (wo = w2 = 0), which makes loss0 independent of the layer count.
The sweep rows also carry the recorded loss after the 10-step protocol
(`loss10`, bench_param_sweep.rs:85-101), which depends on the training math.
"""
from __future__ import annotations

import json
import re
import sys
from pathlib import Path

OUT = Path(__file__).resolve().parent / "published_losses.json"


def parse(root: Path) -> list[dict]:
    rows = []
    sweep = root / "results" / "2026-03-18_1830_param-sweep.md"
    for ln, line in enumerate(sweep.read_text().splitlines(), start=1):
        cells = [c.strip().strip("*") for c in line.strip().strip("|").split("|")]
        if len(cells) < 16 or not re.match(r"^\d", cells[2] or ""):
            continue
        try:
            name = cells[0].split(" ")[0]
            dim, hidden, heads, layers, seq = (int(cells[i]) for i in (2, 3, 4, 5, 6))
            loss0, loss10 = float(cells[13]), float(cells[14])
        except ValueError:
            continue
        rows.append(dict(name=name, dim=dim, hidden=hidden, heads=heads, nlayers=layers, seq=seq, loss0=loss0,
                         loss10=loss10, decimals=3, source=f"results/2026-03-18_1830_param-sweep.md:{ln}"))
    readme = (root / "README.md").read_text().splitlines()
    for ln, line in enumerate(readme, start=1):
        m = re.search(r"Forward pass\.\.\. loss=(\d+\.\d{4})", line)
        if m:
            rows.append(dict(name="600m-A", dim=1536, hidden=4096, heads=12, nlayers=20, seq=512,
                             loss0=float(m.group(1)), decimals=4, source=f"README.md:{ln}"))
        m = re.search(r"Training 10 steps\.\.\. (\d+\.\d{4}) → (\d+\.\d{4})", line)
        if m:
            rows.append(dict(name="600m-A", dim=1536, hidden=4096, heads=12, nlayers=20, seq=512,
                             loss0=float(m.group(1)), loss10=float(m.group(2)), decimals=4, source=f"README.md:{ln}"))
        m = re.search(r"\(loss=(\d+\.\d{4})\)", line)
        if m and "ms" in line:
            rows.append(dict(name="7B", dim=4096, hidden=11008, heads=32, nlayers=32, seq=512,
                             loss0=float(m.group(1)), decimals=4, source=f"README.md:{ln}"))
    return rows


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: python tests/golden/extract_published.py <reference-root>")
    root = Path(sys.argv[1])
    rows = parse(root)
    OUT.write_text(json.dumps(rows, indent=1) + "\n")
    print(f"wrote {len(rows)} rows to {OUT}")
