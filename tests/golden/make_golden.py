"""Regenerate tests/golden/*.npz from the NeuralSuite reference itself.

Runs the reference (oracle/_ref/libnsref.so, compiled from the reference's own
sources by oracle/Makefile) on small seeded inputs and stores inputs and
outputs.  The fixtures pin the C restatement (oracle/ns_oracle.c) bit for bit
on machines where the reference sources are not available.

    python tests/golden/make_golden.py
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))

import oracle  # noqa: E402

GPT_CASES = {
    # include/gpt.h weight-tying test config, test_suite.cpp:230-273
    "gpt_tiny": dict(V=11, block=6, L=2, H=2, C=8, B=2, T=5, steps=3),
    # byte vocabulary, two blocks
    "gpt_small": dict(V=256, block=16, L=2, H=2, C=32, B=2, T=16, steps=2),
}

MHA_CASES = {  # (B, T, E, H) from test_suite.cpp:3112-3119
    "mha_min": (1, 8, 16, 2),
    "mha_one_head": (2, 5, 4, 1),
    "mha_eight_heads": (3, 16, 32, 8),
    "mha_one_token": (1, 1, 8, 2),
}


def gpt_params(g, r):
    parts = []
    n_t = g.num_tensors()
    for i in range(n_t):
        k = g.tensor_numel(i)
        if g.tensor_rank(i) == 2:
            parts.append((r.standard_normal(k) * 0.02).astype(np.float32))
        else:
            parts.append((r.standard_normal(k) * 0.1).astype(np.float32))
    return np.concatenate(parts)


def main():
    oracle.build(ref=True)
    R = oracle.ref()
    r = np.random.default_rng(20261201)
    out = {}
    A = r.standard_normal((7, 5)).astype(np.float32)
    B = r.standard_normal((5, 6)).astype(np.float32)
    out["matmul"] = dict(A=A, B=B, C=R.matmul(A, B))
    x = (r.standard_normal((13, 40)) * 2 + 0.5).astype(np.float32)
    g = (r.standard_normal(40) + 1).astype(np.float32)
    b = r.standard_normal(40).astype(np.float32)
    d = r.standard_normal((13, 40)).astype(np.float32)
    o, m, s = R.layernorm_fwd(x, g, b)
    dx, dg, db = R.layernorm_bwd(d, x, g, m, s)
    out["layernorm"] = dict(x=x, g=g, b=b, dout=d, out=o, mean=m, rstd=s, dx=dx, dg=dg, db=db)
    v = (r.standard_normal(257) * 3).astype(np.float32)
    dv = r.standard_normal(257).astype(np.float32)
    out["gelu"] = dict(x=v, dout=dv, y=R.gelu_fwd(v), dx=R.gelu_bwd(dv, v))
    lg = (r.standard_normal((17, 11)) * 2).astype(np.float32)
    t = r.integers(0, 11, 17).astype(np.float32)
    loss, dl = R.cross_entropy(lg, t)
    out["cross_entropy"] = dict(logits=lg, targets=t, loss=np.array([loss], np.float32), dlogits=dl)
    w = (r.standard_normal((11, 8)) * 0.02).astype(np.float32)
    idx = r.integers(0, 11, (2, 5)).astype(np.float32)
    dd = r.standard_normal((2, 5, 8)).astype(np.float32)
    eo, edw = R.embedding(w, idx, dd)
    out["embedding"] = dict(w=w, idx=idx, dout=dd, out=eo, dw=edw)
    for name, (Bb, T, E, H) in MHA_CASES.items():
        ws = [(r.standard_normal(s) * 0.1).astype(np.float32) for s in [(E, 3 * E), (3 * E,), (E, E), (E,)]]
        xx = (r.standard_normal((Bb, T, E)) * 0.5).astype(np.float32)
        do = r.standard_normal((Bb, T, E)).astype(np.float32)
        y, dxx, gr = R.mha(Bb, T, E, H, *ws, xx, do)
        out[name] = dict(shape=np.array([Bb, T, E, H]), w_attn=ws[0], b_attn=ws[1], w_proj=ws[2],
                         b_proj=ws[3], x=xx, dout=do, y=y, dx=dxx, g_w_attn=gr[0], g_b_attn=gr[1],
                         g_w_proj=gr[2], g_b_proj=gr[3])
    for name, c in GPT_CASES.items():
        gm = R.gpt(c["V"], c["block"], c["L"], c["H"], c["C"])
        p0 = gpt_params(gm, r)
        gm.set_params(p0)
        gm.adamw_init(3e-4)
        idx = r.integers(0, c["V"], (c["B"], c["T"])).astype(np.float32)
        tg = r.integers(0, c["V"], c["B"] * c["T"]).astype(np.float32)
        losses, grads0, logits0 = [], None, None
        for s in range(c["steps"]):
            l, lgt = gm.fwd_bwd(idx, tg)
            losses.append(l)
            if s == 0:
                grads0, logits0 = gm.get_grads(), lgt
            gm.adamw_step()
        out[name] = dict(cfg=np.array([c[k] for k in ("V", "block", "L", "H", "C", "B", "T", "steps")]),
                         params0=p0, idx=idx, targets=tg, loss0=np.array([losses[0]], np.float32),
                         losses=np.array(losses, np.float32), logits0=logits0, grads0=grads0,
                         params_final=gm.get_params())
    for name, arrays in out.items():
        np.savez_compressed(os.path.join(HERE, name + ".npz"), **arrays)
        print(name, sum(a.nbytes for a in arrays.values()), "bytes")


if __name__ == "__main__":
    main()
