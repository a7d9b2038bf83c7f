"""CPU: the mixture-of-experts pieces of the oracle (the checker of the
config-4 GPU tests) against direct restatements — softmax top-k routing with
ties to the lower expert and weights renormalised over the k, one expert as
down(H32(silu(gate) * up)) on the dense linear, and the combine's two fp16
roundings."""
import numpy as np

import r4q_oracle as O


def test_route_matches_bruteforce_and_ties():
    rng = np.random.default_rng(0)
    B, E, k = 9, 16, 4
    lg = rng.standard_normal((B, E)).astype(np.float16)
    lg[0, 3] = lg[0, 7] = lg[0, 11] = np.float16(4.0)          # three-way tie at the top
    ids, w = O.moe_route(lg, k)
    for b in range(B):
        x = lg[b].astype(np.float64)
        order = sorted(range(E), key=lambda e: (-x[e], e))[:k]   # value desc, then lower index
        assert list(ids[b]) == order
        p = np.exp(x - x.max())
        p /= p.sum()
        sel = p[order]
        assert np.allclose(w[b], sel / sel.sum(), rtol=1e-12, atol=0)
        assert abs(w[b].sum() - 1.0) < 1e-12
    assert list(ids[0][:3]) == [3, 7, 11]


def test_expert_is_down_of_silu_fwht_of_gate_up():
    rng = np.random.default_rng(1)
    D, Ie = 64, 64
    x = rng.standard_normal(D).astype(np.float16)
    Wgu = (rng.standard_normal((2 * Ie, D)) * 0.05).astype(np.float16)
    Wd = (rng.standard_normal((D, Ie)) * 0.05).astype(np.float16)
    y = O.moe_expert(x, ('fp16', Wgu), ('fp16', Wd), Ie)
    g = O.linear(x[None], ('fp16', Wgu))
    act = O.silu_fwht(g[:, :Ie], g[:, Ie:])
    assert np.array_equal(y, O.linear(act, ('fp16', Wd))[0])
    # silu * up then the normalised H32 butterfly: orthogonal, so the norm of
    # the activation block is kept up to fp16 rounding
    gf, uf = g[0, :Ie].astype(np.float64), g[0, Ie:].astype(np.float64)
    v = gf / (1 + np.exp(-gf)) * uf
    assert np.allclose(np.linalg.norm(act.astype(np.float64)), np.linalg.norm(v), rtol=2e-3)


def test_combine_rounds_the_sum_then_the_residual_add():
    rng = np.random.default_rng(2)
    k, D = 8, 32
    ys = rng.standard_normal((k, D)).astype(np.float16)
    w = rng.random(k)
    w /= w.sum()
    r = rng.standard_normal(D).astype(np.float16)
    h = O.moe_combine(ys, w, r)
    s16 = (w[:, None] * ys.astype(np.float64)).sum(0).astype(np.float16)
    assert np.array_equal(h, (s16.astype(np.float32) + r.astype(np.float32)).astype(np.float16))
