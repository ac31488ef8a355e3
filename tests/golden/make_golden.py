"""Regenerates the committed fixtures under tests/golden/ from the oracle.

    python tests/golden/make_golden.py

philox_u32.json  -- raw Philox2x32-10 words of the restated generator
                    (Philox.java:41-78) for paths and seeds that exercise the
                    high 32 bits, several streams and pair counters; the GPU
                    test checks the device words against it bit for bit.
oracle_cases.json -- small replays (sums of every channel, exact summation)
                    that the GPU parity tests compare against without having
                    to rerun the oracle.
The reference publishes no uint32 vector, so the words come from the
restatement, which is itself pinned by the published golden prices
(reference_docs.json, tests/test_oracle_golden.py).
"""
import json
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

from oracle import oracle as O  # noqa: E402

ATM = [100.0, 100.0, 0.20, 0.03, 1.0]


def philox_cases():
    cases = []
    for path, seed, stream in [(0, 42, 0), (1, 42, 0), (0x1_0000_0003, 0x1234_5678_FEDC_BA98, 0),
                               (0xFFFF_FFFF, 0xFFFF_FFFF_FFFF_FFFF, 0), (123_456_789, 7, 1),
                               (2**63 + 5, 2**40 + 11, 5), (999, 0xC0FFEE, 2)]:
        pair0 = 0 if stream == 0 else 3
        words = [list(O.normal_words(path, seed, stream, pair0 + q)) for q in range(130)]
        cases.append({"path": path, "seed": seed, "stream": stream, "pair0": pair0, "words": words})
    return {"generator": "Philox2x32-10, key 0x1BD11BDA, Philox.java:41-78", "cases": cases}


def oracle_cases():
    out = []
    specs = [
        ("asian", 64, 20_000, 0x1_0000_0003, 20260830),
        ("asian", 252, 20_000, 0, 42),
        ("asian", 252, 513, 0x1_0000_0003, 0x1234_5678_FEDC_BA98),
        ("barrier_di", 252, 20_000, 0, 42),
        ("european", 1, 200_000, 0, 20260830),
    ]
    for kind, steps, paths, off, seed in specs:
        if kind == "asian":
            t = O.asian_tape(steps)
        elif kind == "european":
            t = O.european_tape(steps)
        else:
            t = O.barrier_tape(steps, True, "DOWN_IN", 80.0, 1.0)
        r = O.replay(t, ATM, paths, off, seed, exact=True)
        out.append({"kind": kind, "steps": steps, "paths": paths, "path_offset": off, "seed": seed,
                    "inputs": ATM, "sums": list(map(float, r.sums))})
    return {"summation": "exact (compensated) sums of the oracle's per-path values", "cases": out}


if __name__ == "__main__":
    with open(os.path.join(HERE, "philox_u32.json"), "w") as f:
        json.dump(philox_cases(), f, separators=(",", ":"))
    with open(os.path.join(HERE, "oracle_cases.json"), "w") as f:
        json.dump(oracle_cases(), f, indent=1)
    print("wrote", os.listdir(HERE))
