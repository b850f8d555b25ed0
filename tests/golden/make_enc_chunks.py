"""Generate tests/golden/enc_chunks.json: the reference's own encoder token
counts for a set of mel frame counts.

Needs the reference sources (read where they lie, never copied here):
    make -C oracle ref && python tests/golden/make_enc_chunks.py

oracle/_ref/enc_tokens_ref is the reference's compute_causal_conv1d_dims,
mel_frames_to_enc_tokens and compute_total_enc_tokens (src/voxtral.cpp
:1274-1325) compiled with oracle/enc_tokens_harness.cpp.  The fixture pins
the oracle's restatement of the realtime encoder's chunk geometry.
"""
from __future__ import annotations

import json
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
BIN = os.path.join(HERE, "..", "..", "oracle", "_ref", "enc_tokens_ref")


def frame_counts() -> list[int]:
    edges = list(range(0, 12)) + [99, 100, 101, 749, 750, 751, 1499, 1500, 1501, 1502, 1503]
    for base in (3000, 4500, 6000, 7500, 60000):       # chunk and stride boundaries, 10 min of audio
        edges += list(range(base - 4, base + 5))
    rng = np.random.default_rng(2024)
    edges += [int(x) for x in rng.integers(12, 400_000, 200)]   # up to ~67 min of audio
    return sorted(set(edges))


def main() -> None:
    counts = frame_counts()
    out = subprocess.run([BIN], input="\n".join(map(str, counts)) + "\n", capture_output=True, text=True,
                         check=True).stdout
    rows = [[int(t) for t in line.split()] for line in out.strip().splitlines()]
    assert [r[0] for r in rows] == counts
    with open(os.path.join(HERE, "enc_chunks.json"), "w") as f:
        json.dump({"source": "reference src/voxtral.cpp:1274-1325 compiled by `make -C oracle ref`",
                   "columns": ["mel_frames", "mel_frames_to_enc_tokens", "compute_total_enc_tokens"],
                   "rows": rows}, f, separators=(",", ":"))
        f.write("\n")
    print(f"wrote {len(rows)} rows")


if __name__ == "__main__":
    main()
