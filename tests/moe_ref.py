"""fp64-oracle references for full-size MoE checks on sampled tokens.

A full-size layer (config 4: 64 experts x 3 matrices of 2048 x 1408; config 5: 8 experts x 3
matrices of 4096 x 14336) is too large to dequantise whole on the host. The sampled tokens'
routed experts are dequantised one at a time on the device (ckl_moe_dequant_weights over a
one-expert view: the same bit-exact (q - z) * s values the layer multiplies by), and the
oracle (oracle/ckl_oracle.cpp ora_moe_layer, the fp64 restatement of 03_moe_wq_decode.cu:
471-479 extended with SwiGLU) computes every routed row in fp64; the k rows of a token are
then combined in fixed slot order with the oracle's fp64 routing weights (the reference's
moe_combine order, common/moe.cuh:97-119).
"""
import numpy as np


def rel_rms(got, ref):
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    return float(np.linalg.norm(got - ref) / max(np.linalg.norm(ref), 1e-30))


def sample_tokens(T, n=8, seed=0):
    """All tokens when T <= n, else n distinct tokens (first and last included)."""
    if T <= n:
        return list(range(T))
    rng = np.random.default_rng(seed + T)
    mid = rng.choice(np.arange(1, T - 1), size=n - 2, replace=False)
    return sorted({0, T - 1, *mid.tolist()})


def sampled_layer_ref(oracle, logits, X, k, gate, up, down, tokens):
    """fp64 layer output [len(tokens), d] for the sampled tokens, and the oracle's routing
    ids [T, k] of the whole batch. logits fp32 [T, E] and X fp16 [T, d] are host arrays;
    gate/up/down are ckl.QuantWeights on the device."""
    rids, rwts = oracle.route(np.ascontiguousarray(logits, np.float32), k)
    d = down.N
    ys = {}                                        # (token index, slot) -> fp64 row
    by_expert = {}
    for ti, t in enumerate(tokens):
        for j in range(k):
            by_expert.setdefault(int(rids[t, j]), []).append((ti, t, j))
    for e, rows in sorted(by_expert.items()):
        Wg = gate.expert(e).dequant().cpu().numpy()
        Wu = up.expert(e).dequant().cpu().numpy()
        Wd = down.expert(e).dequant().cpu().numpy()
        Xe = np.ascontiguousarray(X[[t for _, t, _ in rows]], np.float16)
        n = len(rows)
        y = oracle.moe_layer(Xe, np.zeros((n, 1), np.int32), np.ones((n, 1), np.float64),
                             Wg, Wu, Wd)
        for r, (ti, _, j) in enumerate(rows):
            ys[(ti, j)] = y[r].astype(np.float64)
        del Wg, Wu, Wd
    out = np.zeros((len(tokens), d), np.float64)
    for ti, t in enumerate(tokens):
        for j in range(k):
            out[ti] += rwts[t, j] * ys[(ti, j)]
    return out, rids
