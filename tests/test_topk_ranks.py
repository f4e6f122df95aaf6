"""The routing kernel's single-token top-k counts ranks instead of running the
reference's n_used rounds of warp argmax (src/fr_win_qwen36_sm120.cu:1826-1870).
This pins, on the CPU, that the restatement picks the same experts in the same
order and produces the same weight bits, with ties (to the lower id) and NaN
probabilities (read as -FLT_MAX) included:

  * rounds: each round takes the largest remaining probability, ties to the
    lower expert id; the winner's lane (id % 32) adds it to its partial sum;
  * ranks: expert e is picked in round r = #{e' : p[e'] > p[e] or
    (p[e'] == p[e] and e' < e)}; lane L adds its winners in round order;
  * both: the 32 lane partials summed by the xor butterfly, max(sum, clamp),
    weights p * (1 / sum), all in fp32.
"""
import numpy as np
import pytest

FLT_MAX = np.float32(np.finfo(np.float32).max)


def _butterfly(parts):
    v = parts.astype(np.float32).copy()
    for off in (16, 8, 4, 2, 1):
        v = (v + v[np.arange(32) ^ off]).astype(np.float32)
    return v


def _rounds(p, n_used, clamp):
    wt = p.copy()
    ids, vals = [], []
    parts = np.zeros(32, np.float32)
    for _ in range(n_used):
        e = int(np.argmax(wt))                       # first maximum: ties to the lower id
        ids.append(e)
        vals.append(wt[e])
        parts[e & 31] = np.float32(parts[e & 31] + wt[e])
        wt[e] = -np.inf
    s = np.maximum(_butterfly(parts), np.float32(clamp))
    inv = (np.float32(1.0) / s).astype(np.float32)
    return np.array(ids), np.array([np.float32(v * inv[k]) for k, v in enumerate(vals)], np.float32)


def _ranks(p, n_used, clamp):
    E = p.size
    idx = np.arange(E)
    rank = np.array([int(np.sum(p > p[e]) + np.sum((p == p[e]) & (idx < e))) for e in range(E)])
    parts = np.zeros(32, np.float32)
    for r in range(n_used):
        e = int(np.nonzero(rank == r)[0][0])
        parts[e & 31] = np.float32(parts[e & 31] + p[e])
    s = np.maximum(_butterfly(parts), np.float32(clamp))
    inv = (np.float32(1.0) / s).astype(np.float32)
    ids = np.empty(n_used, np.int64)
    w = np.empty(n_used, np.float32)
    for e in range(E):
        if rank[e] < n_used:
            ids[rank[e]] = e
            w[rank[e]] = np.float32(p[e] * inv[rank[e]])
    return ids, w


@pytest.mark.parametrize("E,n_used", [(32, 1), (128, 8), (128, 32), (256, 8), (64, 3)])
def test_ranks_equal_rounds(E, n_used):
    rng = np.random.default_rng(E * 100 + n_used)
    clamp = 6.103515625e-5
    for trial in range(60):
        logits = rng.standard_normal(E).astype(np.float32)
        if trial % 3 == 0:                                   # ties: repeated logits
            logits = np.round(logits * 2).astype(np.float32) / np.float32(2)
        ex = np.exp(logits - logits.max()).astype(np.float32)
        p = (ex * (np.float32(1.0) / ex.sum(dtype=np.float32))).astype(np.float32)
        if trial % 5 == 0:                                   # NaN probabilities read as -FLT_MAX
            p[rng.choice(E, 3, replace=False)] = -FLT_MAX
        if trial % 7 == 0:                                   # a block of exact ties at the top
            p[rng.choice(E, min(E, n_used + 2), replace=False)] = p.max()
        ids_a, w_a = _rounds(p, n_used, clamp)
        ids_b, w_b = _ranks(p, n_used, clamp)
        np.testing.assert_array_equal(ids_a, ids_b)
        np.testing.assert_array_equal(w_a.view(np.uint32), w_b.view(np.uint32))


def test_ranks_match_oracle_ids(O):
    """On probabilities the oracle's own top-k sees (fp32 softmax of fp32
    logits), the rank selection gives the oracle's ids."""
    rng = np.random.default_rng(7)
    E, n_used = 128, 8
    logits = rng.standard_normal((16, E)).astype(np.float32)
    logits[3, :40] = logits[3, 0]                            # ties across lanes
    ids_o, _ = O.topk_softmax(logits, n_used)
    for t in range(logits.shape[0]):
        ex = np.exp((logits[t] - logits[t].max()).astype(np.float32)).astype(np.float32)
        p = (ex * (np.float32(1.0) / ex.sum(dtype=np.float32))).astype(np.float32)
        ids_r, _ = _ranks(p, n_used, 6.103515625e-5)
        np.testing.assert_array_equal(ids_r, ids_o[t])
