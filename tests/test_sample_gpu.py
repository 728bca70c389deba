"""Token sampling on the GPU (mmrs_sample_token, mmrs_token_logprob) against the CPU oracle
(oracle/sample_oracle.c, a restatement of src/sampling.rs) on the model's vocabulary of 200064
ids.  The token must equal the oracle's for the same draw u whenever the oracle's margin (how close
a compared sum came to its bound) is above rounding level; draws closer than that are skipped
(none are expected at these sizes)."""
from __future__ import annotations

import numpy as np
import pytest

V = 200064
MARGIN = 1e-9

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def logits_np():
    return (np.random.default_rng(7001).standard_normal(V) * 4.0).astype(np.float32)


def _nucleus_len(x: np.ndarray, top_k: int, top_p: float) -> int:
    k = top_k if 0 < top_k < x.size else x.size
    s = np.sort(x.astype(np.float64))[::-1][:k]
    w = np.exp(s - s[0])
    return int(np.searchsorted(np.cumsum(w), w.sum() * top_p) + 1)


def _check(pkg, orc, sampler_dev, x_np, x_dev, t, p, k, draws):
    s = pkg.Sampler(x_np.size, sampler_dev, temperature=t, top_p=p, top_k=k)
    too_long = t > 0 and p < 1.0 and (k == 0 or k > 1024) and _nucleus_len(x_np, k, p) > 1024
    checked = 0
    for u in draws:
        tok = int(s.sample(x_dev, float(u)).item())
        if too_long:
            assert tok == -1 and s.status() == pkg.MMRS_ERR_UNSUPPORTED
            continue
        st, want, margin = orc.sample_token(x_np, t, p, k, float(u))
        assert st == 0 and s.status() == pkg.MMRS_OK
        if margin > MARGIN:
            assert tok == want, (t, p, k, u, margin)
            checked += 1
    return checked


@pytest.mark.parametrize("t", [0.7, 1.0, 1.5])
@pytest.mark.parametrize("k,p", [(40, 0.95), (1, 1.0), (40, 1.0), (1024, 0.9), (1024, 1.0), (0, 1.0),
                                 (5000, 0.9), (5000, 1.0), (0, 0.9), (2, 0.0), (7, 0.5)])
def test_sample_matches_oracle(pkg, orc, dev, logits_np, t, k, p):
    import torch
    x = torch.from_numpy(logits_np).to(dev)
    draws = np.random.default_rng(int(t * 100) + 7 * k + int(p * 1000)).random(6)
    draws[0] = 0.0
    _check(pkg, orc, dev, logits_np, x, t, p, k, draws)


def test_greedy_matches_lm_head_choice(pkg, orc, dev, logits_np):
    import torch
    x = torch.from_numpy(logits_np).to(dev)
    s = pkg.Sampler(V, dev, temperature=0.0)
    assert int(s.sample(x).item()) == orc.argmax_f32(logits_np)


def test_ties_and_signed_zero(pkg, orc, dev):
    """Many equal logits: compare_candidates puts the lower id first; total_cmp puts -0 below +0."""
    import torch
    rng = np.random.default_rng(7002)
    x = np.round(rng.standard_normal(V) * 1.5).astype(np.float32)
    x[rng.integers(0, V, 500)] = -0.0
    xd = torch.from_numpy(x).to(dev)
    for t, p, k in ((1.0, 0.9, 40), (1.0, 0.5, 1024), (1.0, 1.0, 300), (0.5, 0.2, 1000), (2.0, 1.0, 0)):
        _check(pkg, orc, dev, x, xd, t, p, k, rng.random(4))
    y = np.zeros(64, np.float32)
    y[::2] = -0.0
    for u in (0.0, 0.3, 0.99):  # top-1 of all zeros: +0 beats -0, then the lower id
        _check(pkg, orc, dev, y, torch.from_numpy(y).to(dev), 1.0, 0.0, 5, [u])


def test_reference_unit_cases_on_gpu(pkg, dev):
    """src/sampling.rs:205-252 through the device path."""
    import torch
    a = torch.tensor([0.0, 3.0, 2.0], device=dev)
    assert int(pkg.Sampler(3, dev, temperature=0.0, top_p=0.01, top_k=1).sample(a).item()) == 1
    s = pkg.Sampler(3, dev, temperature=100.0, top_p=1.0, top_k=1)
    assert all(int(s.sample(a, u).item()) == 1 for u in np.random.default_rng(3).random(16))
    b = torch.tensor([3.0, 2.0, 1.0, 0.0], device=dev)
    s = pkg.Sampler(4, dev, temperature=1.0, top_p=0.7, top_k=3)
    got = {int(s.sample(b, u).item()) for u in np.random.default_rng(4).random(64)}
    assert got == {0, 1}
    with pytest.raises(pkg.MoeError):
        pkg.Sampler(3, dev, temperature=-0.1)
    with pytest.raises(pkg.MoeError):
        pkg.Sampler(3, dev, top_p=1.1)


def test_non_finite_and_recovery(pkg, dev, logits_np, orc):
    """Non-finite logits: MMRS_ERR_NONFINITE and token -1 (greedy still answers); an over-long
    nucleus: MMRS_ERR_UNSUPPORTED; the same workspace then serves ordinary calls."""
    import torch
    s = pkg.Sampler(V, dev, temperature=1.0, top_p=0.95, top_k=40)
    bad = logits_np.copy()
    bad[12345] = np.nan
    assert int(s.sample(torch.from_numpy(bad).to(dev), 0.5).item()) == -1
    assert s.status() == pkg.MMRS_ERR_NONFINITE
    bad[12345] = np.inf
    assert int(s.sample(torch.from_numpy(bad).to(dev), 0.5).item()) == -1
    g = pkg.Sampler(V, dev, temperature=0.0)
    assert int(g.sample(torch.from_numpy(bad).to(dev)).item()) == 12345
    flat = (np.random.default_rng(7003).standard_normal(V) * 0.1).astype(np.float32)
    s2 = pkg.Sampler(V, dev, temperature=1.0, top_p=0.95, top_k=0)
    s2.ws = s.ws  # one workspace through every outcome
    assert int(s2.sample(torch.from_numpy(flat).to(dev), 0.5).item()) == -1
    assert s2.status() == pkg.MMRS_ERR_UNSUPPORTED
    x = torch.from_numpy(logits_np).to(dev)
    for u in (0.1, 0.6, 0.95):
        want = orc.sample_token(logits_np, 1.0, 0.95, 40, u)[1]
        assert int(s.sample(x, u).item()) == want and s.status() == pkg.MMRS_OK
    with pytest.raises(pkg.MoeError):
        s.sample(x, 1.0)  # the draw must lie in [0, 1)


def test_repeatable(pkg, dev, logits_np):
    import torch
    x = torch.from_numpy(logits_np).to(dev)
    s = pkg.Sampler(V, dev, temperature=1.0, top_p=1.0, top_k=0)
    a = [int(s.sample(x, u).item()) for u in np.linspace(0.0, 0.999, 25)]
    b = [int(s.sample(x, u).item()) for u in np.linspace(0.0, 0.999, 25)]
    assert a == b


def test_token_logprob(pkg, orc, dev, logits_np):
    import torch
    x = torch.from_numpy(logits_np).to(dev)
    s = pkg.Sampler(V, dev)
    for t in (0, 1, int(np.argmax(logits_np)), V - 1, 99999):
        got = float(s.token_logprob(x, t).item())
        st, want = orc.token_logprob(logits_np, t)
        assert st == 0 and s.status() == pkg.MMRS_OK and abs(got - want) <= 1e-5 * max(1.0, abs(want))
    small = torch.tensor([0.0, float(np.log(3.0))], device=dev)
    s2 = pkg.Sampler(2, dev)
    assert abs(float(s2.token_logprob(small, 0).item()) - np.log(0.25)) < 1e-6
    assert abs(float(s2.token_logprob(small, 1).item()) - np.log(0.75)) < 1e-6
    with pytest.raises(pkg.MoeError):
        s2.token_logprob(small, 2)
    s2.token_logprob(torch.tensor([0.0, float("inf")], device=dev), 0)
    assert s2.status() == pkg.MMRS_ERR_NONFINITE
