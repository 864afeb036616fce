"""Generates the committed golden fixtures from the reference engine's own C
attention (oracle/_ref/libndref.so, compiled from engine/src/nd_model.c).

Run from the repository root where the reference sources are present:
    python tests/golden/make_golden.py

Fixtures (inputs are regenerated from the seeds, so only outputs are stored):
  config1_int8.npz  config 1 of the benchmark set: one sequence, 213-token prefix pinned as
                    sinks (nd_model_set_sink), 40-token suffix, 32 decode steps;
                    8 q / 8 kv heads x 64, theta 1e4, q/k/v ~ N(0,1)*0.5 seed 0,
                    no gate. The reference's only KV format is int8.
  model48_int8.npz  the reference model's own attention geometry
                    (engine docs: 12 q / 2 kv heads, qk 48, v 64, theta 1e5,
                    window 384) with per-head norms and gates, 2 layers, a
                    40-token prefix pinned, 30 more tokens; seed 11.
Each stores: out [tokens][H*VD] f32 for the post-prefix tokens, the final
int8 caches' sha256, the scales, and the sha256 of the saved-prefix image.
"""
import hashlib
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "..", "..", "oracle"))
import ndoracle as O  # noqa: E402

CASES = {
    "config1_int8": dict(H=8, HKV=8, QK=64, VD=64, W=384, L=1, theta=10000.0, prefix=213, tokens=72,
                         seed=0, norm=False, gate=False),
    "model48_int8": dict(H=12, HKV=2, QK=48, VD=64, W=384, L=2, theta=100000.0, prefix=40, tokens=30,
                         seed=11, norm=True, gate=True),
}


def inputs(c):
    """Seeded inputs of a case: q/k/v [tok][layer][...] ~ N(0,1)*0.5, optional norms and gates."""
    rng = np.random.default_rng(c["seed"])
    n = c["prefix"] + c["tokens"]
    q = (rng.standard_normal((n, c["L"], c["H"] * c["QK"])) * 0.5).astype(np.float32)
    k = (rng.standard_normal((n, c["L"], c["HKV"] * c["QK"])) * 0.5).astype(np.float32)
    v = (rng.standard_normal((n, c["L"], c["HKV"] * c["VD"])) * 0.5).astype(np.float32)
    norms = None
    if c["norm"]:
        norms = [((rng.standard_normal(c["QK"]) * 0.1).astype(np.float32),
                  (rng.standard_normal(c["QK"]) * 0.1).astype(np.float32)) for _ in range(c["L"])]
    gate = (rng.standard_normal((n, c["L"], c["H"] * c["VD"]))).astype(np.float32) if c["gate"] else None
    return q, k, v, norms, gate


def run(seq_cls, c, kv_dtype=O.I8):
    q, k, v, norms, gate = inputs(c)
    s = seq_cls(c["L"], c["H"], c["HKV"], c["QK"], c["VD"], c["W"], kv_dtype, theta=c["theta"],
                max_pos=c["W"])
    if norms:
        for l, nv in enumerate(norms):
            s.norms[l] = nv
    outs, prefix_img = [], None
    for t in range(c["prefix"] + c["tokens"]):
        if t == c["prefix"]:
            # The reference's own nd_model_snapshot + nd_model_prefix_save image
            # when running the reference; the restated image otherwise.
            prefix_img = s.ref_prefix_image()[0] if hasattr(s, "ref_prefix_image") else None
            s.snapshot()                       # pins the prefix as sinks
            if prefix_img is None:
                prefix_img = s.prefix_image()
        row = []
        for l in range(c["L"]):
            o = s.step(l, q[t, l], k[t, l], v[t, l], None if gate is None else gate[t, l])
            row.append(np.asarray(o, dtype=np.float64).reshape(-1))
        if t >= c["prefix"]:
            outs.append(np.stack(row))
        s.advance()
    return s, np.stack(outs), prefix_img


def sha(b):
    return hashlib.sha256(b).hexdigest()


def main():
    for name, c in CASES.items():
        s, out, img = run(O.RefSeq, c)
        np.savez_compressed(os.path.join(HERE, name + ".npz"), out=out.astype(np.float32),
                            k_sha=sha(s.k.tobytes()), v_sha=sha(s.v.tobytes()), ks=s.ks, vs=s.vs,
                            prefix_sha=sha(img), sink=np.uint32(min(c["prefix"], c["W"] - 64)))
        print(name, out.shape, "written")


if __name__ == "__main__":
    main()
