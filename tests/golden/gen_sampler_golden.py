"""Generate tests/golden/sampler_golden.npz from the reference's own sampler.

The reference sampler (gsv.cpp src/gsv_sampler.cpp) is compiled in place from the read-only
reference tree into oracle/_ref/libgsv_sampler_ref.so by `make -C oracle ref`. This script feeds it
seeded logits / repetition windows / settings and records its probabilities, sampled tokens and RNG
states. Run from the repository root: python tests/golden/gen_sampler_golden.py
"""
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
import oracle as O  # noqa: E402


def cases(rng, n):
    V = 1025
    for i in range(n):
        scale = [0.1, 0.45, 3.0][i % 3]
        lg = (rng.standard_normal(V) * scale).astype(np.float32)
        if i % 4 == 1:
            lg = (np.round(lg * 8) / 8).astype(np.float32)   # exact ties
        if i % 5 == 2:
            lg[1024] = -np.inf                               # EOS masked (step < 11)
        top_k = [15, 15, 1, 0, 50, 1025][i % 6]
        top_p = [1.0, 1.0, 0.9, 0.5, 1.0, 0.97][i % 6]
        temp = [1.0, 0.7, 1.0, 1.3, 1e-6, 1.0][i % 6]
        rep = [1.35, 1.35, 1.0, 2.0, 1.35, 1.35][i % 6]
        n_prev = int(rng.integers(0, 400))
        prev = rng.integers(0, V, n_prev, dtype=np.int32)
        if i % 3 == 0:
            prev = np.concatenate([prev, np.full(9, 7, np.int32)])   # compounding repeats
        seed = int(rng.integers(1, 2**63))
        yield lg, prev, (top_k, top_p, temp, rep), seed


def main():
    ref = O.RefSampler()
    rng = np.random.default_rng(20261201)
    L, P, NP, CFG, SEED, PROBS, TOK, STATE = [], [], [], [], [], [], [], []
    for lg, prev, cfg, seed in cases(rng, 36):
        probs = ref.logits_to_probs(lg, top_k=cfg[0], top_p=cfg[1], temperature=cfg[2], rep=cfg[3], prev=prev)
        st0 = ref.rng_init(seed)
        tok, st1 = ref.sample(probs, st0)
        pv = np.full(420, -1, np.int32)
        pv[:prev.size] = prev
        L.append(lg); P.append(pv); NP.append(prev.size); CFG.append(cfg); SEED.append(st0)
        PROBS.append(probs); TOK.append(tok); STATE.append(st1)
    out = os.path.join(ROOT, "tests", "golden", "sampler_golden.npz")
    np.savez_compressed(out, logits=np.array(L), prev=np.array(P), n_prev=np.array(NP, np.int32),
                        cfg=np.array(CFG, np.float64), state0=np.array(SEED, np.uint64),
                        probs=np.array(PROBS), token=np.array(TOK, np.int32), state1=np.array(STATE, np.uint64))
    print("wrote", out, os.path.getsize(out), "bytes")


if __name__ == "__main__":
    main()
