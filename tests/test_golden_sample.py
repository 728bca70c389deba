"""The sampling oracle (oracle/sample_oracle.c) pinned to the reference's own sampler tests
(src/sampling.rs:189-262) and to a second, pure-Python restatement of TokenSampler::sample
(:84-150) on small seeded cases.  CPU only.

The reference's tests draw from StdRng; each expectation below holds for every draw, so the draws
here come from numpy."""
from __future__ import annotations

import math
import struct

import numpy as np
import pytest

ERR_ARG, ERR_NONFINITE = 1, 7


def test_recommended_defaults(pkg):
    """recommended_defaults_are_enabled (:193-203)."""
    assert (pkg.DEFAULT_TEMPERATURE, pkg.DEFAULT_TOP_P, pkg.DEFAULT_TOP_K) == (1.0, 0.95, 40)


def test_zero_temperature_is_greedy(orc):
    """zero_temperature_is_greedy (:205-214)."""
    st, tok, _ = orc.sample_token(np.array([0.0, 3.0, 2.0], np.float32), 0.0, 0.01, 1, 0.5)
    assert (st, tok) == (0, 1)


def test_top_k_one_is_greedy_at_positive_temperature(orc):
    """top_k_one_is_greedy_at_positive_temperature (:224-235)."""
    for u in np.random.default_rng(0).random(16):
        assert orc.sample_token(np.array([0.0, 3.0, 2.0], np.float32), 100.0, 1.0, 1, u)[:2] == (0, 1)


def test_top_p_excludes_tokens_after_the_crossing_candidate(orc):
    """top_p_excludes_tokens_after_the_crossing_candidate (:237-252): within the top three of
    [3, 2, 1, 0] the probabilities are about 0.665, 0.245, 0.090, so top_p = 0.7 keeps ids 0 and 1;
    the draw then splits at 0.665 / 0.910 of the kept mass."""
    logits = np.array([3.0, 2.0, 1.0, 0.0], np.float32)
    seen = set()
    for u in np.random.default_rng(1).random(64):
        st, tok, _ = orc.sample_token(logits, 1.0, 0.7, 3, u)
        assert st == 0 and tok in (0, 1)
        seen.add(tok)
    assert seen == {0, 1}
    split = 1.0 / (1.0 + math.exp(-1.0))  # e^3 / (e^3 + e^2)
    assert orc.sample_token(logits, 1.0, 0.7, 3, split - 1e-9)[1] == 0
    assert orc.sample_token(logits, 1.0, 0.7, 3, split + 1e-9)[1] == 1


def test_invalid_ranges_are_rejected(orc):
    """invalid_ranges_are_rejected (:254-262), plus non-finite parameters (validate, :31-39)."""
    x = np.array([0.0, 1.0], np.float32)
    for t, p in ((-0.1, 0.95), (1.0, 1.1), (float("nan"), 0.95), (1.0, float("inf")), (1.0, -0.01)):
        assert orc.sample_token(x, t, p, 40, 0.5)[0] == ERR_ARG


def test_non_finite_logits_are_rejected(orc):
    """sample (:97-99): non-finite logits fail stochastic decoding, not greedy decoding."""
    for bad in (float("nan"), float("inf"), float("-inf")):
        x = np.array([0.0, bad, 1.0], np.float32)
        assert orc.sample_token(x, 1.0, 0.95, 40, 0.5)[0] == ERR_NONFINITE
    assert orc.sample_token(np.array([0.0, float("nan"), 1.0], np.float32), 0.0, 0.95, 40, 0.5)[:2] == (0, 2)


def test_token_logprob_scores_the_unfiltered_distribution(orc):
    """token_logprob_scores_the_unfiltered_distribution (:216-222)."""
    x = np.array([0.0, math.log(3.0)], np.float32)
    assert abs(orc.token_logprob(x, 0)[1] - math.log(0.25)) < 1e-6
    assert abs(orc.token_logprob(x, 1)[1] - math.log(0.75)) < 1e-6
    assert orc.token_logprob(x, 2)[0] == ERR_ARG
    assert orc.token_logprob(np.array([0.0, float("inf")], np.float32), 0)[0] == ERR_NONFINITE


# ---- a second restatement, in Python, of TokenSampler::sample -------------------------------------

def _total_order(v: float) -> int:
    u = struct.unpack("<I", struct.pack("<f", v))[0]
    return (~u & 0xFFFFFFFF) if u & 0x80000000 else (u | 0x80000000)


def _py_sample(logits, temperature, top_p, top_k, u):
    if temperature == 0.0:
        return int(np.argmax(logits))
    cands = [(i, float(v)) for i, v in enumerate(logits)]
    key = lambda c: (-_total_order(np.float32(c[1])), c[0])  # noqa: E731  compare_candidates
    if 0 < top_k < len(cands):
        cands = sorted(sorted(cands, key=key)[:top_k])  # the top_k, visited by ascending id
    if top_p < 1.0 and len(cands) > 1:
        cands.sort(key=key)
        mx = cands[0][1]
        w = [math.exp(v - mx) for _, v in cands]
        threshold = sum(w) * top_p  # sum() adds left to right, as Iterator::sum
        cum, keep = 0.0, len(cands)
        for i, wi in enumerate(w):
            cum += wi
            if cum >= threshold:
                keep = i + 1
                break
        cands = cands[:max(keep, 1)]
    mx = max(v for _, v in cands)
    w = [math.exp((v - mx) / temperature) for _, v in cands]
    sample = u * sum(w)
    fallback = cands[0][0]
    for (i, _), wi in zip(cands, w):
        if wi > 0.0:
            fallback = i
        if sample < wi:
            return i
        sample -= wi
    return fallback


@pytest.mark.parametrize("case", range(40))
def test_oracle_matches_python_restatement(orc, case):
    rng = np.random.default_rng(100 + case)
    n = int(rng.integers(1, 80))
    x = (rng.standard_normal(n) * rng.choice([0.5, 2.0, 8.0])).astype(np.float32)
    if case % 4 == 0:
        x = np.round(x).astype(np.float32)  # ties: the lower id first
    if case % 7 == 0:
        x[rng.integers(0, n)] = -0.0
    t = float(rng.choice([0.0, 0.3, 1.0, 2.5]))
    p = float(rng.choice([0.0, 0.5, 0.9, 1.0]))
    k = int(rng.choice([0, 1, 3, 17, 200]))
    for u in rng.random(8):
        st, tok, _ = orc.sample_token(x, t, p, k, float(u))
        assert st == 0 and tok == _py_sample(x, t, p, k, float(u)), (t, p, k, u)


def test_host_side_rejections_launch_nothing(pkg):
    """mmrs_sample_token / mmrs_token_logprob check their arguments before any CUDA call
    (SamplingParams::validate, src/sampling.rs:31-39; the draw in [0, 1)), so this runs without a GPU."""
    import ctypes as C
    lib = pkg.lib()
    assert lib.mmrs_sample_workspace_bytes(0) == 0 and lib.mmrs_sample_workspace_bytes(1 << 20 | 1) == 0
    assert lib.mmrs_sample_workspace_bytes(200064) > 0
    fake = C.c_void_p(256)  # never dereferenced: every call below fails validation first
    bad = [(-0.1, 0.95, 40, 0.5), (float("nan"), 0.95, 40, 0.5), (1.0, 1.5, 40, 0.5), (1.0, float("nan"), 40, 0.5),
           (1.0, 0.95, 40, 1.0), (1.0, 0.95, 40, -0.1), (1.0, 0.95, 40, float("nan"))]
    for t, p, k, u in bad:
        prm = pkg.MmrsSamplingParams(t, p, k)
        assert lib.mmrs_sample_token(fake, 200064, C.byref(prm), u, fake, fake, 1 << 20, None) == pkg.MMRS_ERR_ARG
    ok = pkg.MmrsSamplingParams(1.0, 0.95, 40)
    assert lib.mmrs_sample_token(None, 200064, C.byref(ok), 0.5, fake, fake, 1 << 20, None) == pkg.MMRS_ERR_ARG
    assert lib.mmrs_sample_token(fake, 0, C.byref(ok), 0.5, fake, fake, 1 << 20, None) == pkg.MMRS_ERR_ARG
    assert lib.mmrs_token_logprob(fake, 10, 10, fake, fake, 1 << 20, None) == pkg.MMRS_ERR_ARG
    assert lib.mmrs_token_logprob(fake, 10, -1, fake, fake, 1 << 20, None) == pkg.MMRS_ERR_ARG


@pytest.mark.parametrize("x,t,p,k", [
    ([1.5], 1.0, 0.9, 40),                       # one candidate
    ([0.0, 2.0, 1.0], 1.0, 0.95, 10),            # top_k above the vocabulary
    ([0.0, 2.0, 1.0, 2.0], 1e-30, 1.0, 0),       # weights underflow: only the maxima remain
    ([0.0, 2.0, 1.0, 2.0], 1e-30, 0.5, 0),
    ([-3.0, -1.0, -2.0], 0.5, 0.999999, 2),
    ([5.0] * 9, 2.0, 0.3, 4),                    # all equal: lowest ids first
])
def test_oracle_edge_cases_match_python_restatement(orc, x, t, p, k):
    x = np.array(x, np.float32)
    for u in (0.0, 0.25, 0.5, 0.999, 1.0 - 2.0 ** -53):
        st, tok, _ = orc.sample_token(x, t, p, k, u)
        assert st == 0 and tok == _py_sample(x, t, p, k, u), (u, tok)
