"""Regenerate the golden sampling fixtures in this folder (run from the repo root:
``python tests/golden/make_golden.py``).

The reference ships no golden vectors for its sampling path and cannot run in this
image (TypeScript, no Node), so the goldens are produced by the C parity oracle
(oracle/, a restatement of src/engine/sampler.ts:13-30,147-212 pinned against the
reference's known answers in tests/sampling.test.ts:206-250) on the seeded synthetic
configurations of tabby_b200/synth.py. Each case stores the SHA-256 of its generated
logits so a change of the generator is caught instead of silently moving the goldens.
"""
import hashlib
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from oracle import oracle  # noqa: E402
from tabby_b200 import synth  # noqa: E402

# (name, config, seed, rows, top_k override, cap, shards)
CASES = [
    ("c1_k40", "c1", 0, 1, None, 64, 0),
    ("c2_k1", "c2", 0, 1, 1, 64, 0),
    ("c2_k50", "c2", 0, 1, 50, 64, 0),
    ("c3_k1", "c3", 0, 2, 1, 1024, 0),
    ("c3_k8", "c3", 0, 2, 8, 1024, 0),
    ("c3_k64", "c3", 0, 2, 64, 1024, 0),
    ("c3_k256", "c3", 0, 2, 256, 1024, 0),
    ("c3_k1024", "c3", 0, 2, 1024, 1024, 0),
    ("c4_rows6", "c4", 0, 6, None, 1024, 0),
    ("c5_shards2", "c5", 0, 3, None, 64, 2),
    ("c5_shards4", "c5", 0, 3, None, 64, 4),
]


def digest(x: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(x, np.float32).tobytes()).hexdigest()


def inputs(case):
    _, cfg, seed, rows, top_k, _, _ = case
    return synth.config(cfg, seed=seed, rows=rows, top_k=top_k)


def expected(case, x, p, u):
    name, cfg, seed, rows, top_k, cap, shards = case
    if shards:
        V = x.shape[1]
        blocks = [oracle.shard_local_block(x[:, s * V // shards:(s + 1) * V // shards],
                                           s * V // shards) for s in range(shards)]
        return oracle.shard_merge(np.concatenate(blocks, 0), shards, p, u)
    return oracle.sample_rows(x, p, u, cap)


def record(case):
    x, p, u = inputs(case)
    out, ids, vals = expected(case, x, p, u)
    rows = []
    for r in range(x.shape[0]):
        o = out[r]
        n = int(o["pool_size"])
        rows.append(dict(
            id=int(o["id"]), considered_count=int(o["considered_count"]),
            probability=float(o["probability"]), pool_mass=float(o["pool_mass"]),
            pool_exhausted=int(o["pool_exhausted"]), pool_size=n,
            max_logit=float(o["max_logit"]), sum_exp=float(o["sum_exp"]),
            topk_ids=[int(i) for i in ids[r, :n]],
            topk_values_hex=np.ascontiguousarray(vals[r, :n]).view(np.uint32).tobytes().hex(),
            temperature=float(p[r]["temperature"]), top_p=float(p[r]["top_p"]),
            top_k=int(p[r]["top_k"]), uniform=float(u[r])))
    name, cfg, seed, nrows, top_k, cap, shards = case
    return dict(name=name, config=cfg, seed=seed, rows=nrows, top_k=top_k, cap=cap,
                shards=shards, logits_sha256=digest(x), expected=rows)


def main():
    data = dict(generator="tests/golden/make_golden.py", cases=[record(c) for c in CASES])
    path = os.path.join(HERE, "sampling_golden.json")
    with open(path, "w") as f:
        json.dump(data, f, indent=1)
    print(f"wrote {path}")


if __name__ == "__main__":
    main()
