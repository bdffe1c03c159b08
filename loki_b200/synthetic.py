"""Synthetic workload pieces shared by the benchmark and the tests (no GPU work here).

Load-imbalance router bias: expert popularity follows a Zipf law over 256 experts through
the e_score_correction bias, bias_e = lam * (-s * ln(rank_e)) with rank_e a seeded permutation of 1..256,
lam calibrated so that the hottest expert receives about `target` times the mean number of (token, k)
entries.  A true Zipf(1.2) share over 256 experts would make the hottest expert ~65x the mean; the config
asks for ~10x, hence the calibration.
"""
import numpy as np

N_EXPERTS = 256


def zipf_ranks(seed=0x21F):
    return np.random.default_rng(seed).permutation(N_EXPERTS) + 1


def zipf_bias(lam, s=1.2, seed=0x21F):
    return (lam * (-s * np.log(zipf_ranks(seed).astype(np.float64)))).astype(np.float32)


def simulate_counts(bias, keep=2, topk=8, tokens=8000, logit_std=0.02 * np.sqrt(7168.0), seed=7, n_group=1,
                    topk_group=1):
    """Tokens per expert when router logits are i.i.d. N(0, logit_std^2) (W ~ N(0, 0.02), x ~ N(0, 1)):
    sigmoid, + bias, (grouped: only the topk_group groups with the largest top-2 sums) top-k by score,
    keep the `keep` largest probabilities among them."""
    rng = np.random.default_rng(seed)
    p = 1.0 / (1.0 + np.exp(-rng.normal(0.0, logit_std, (tokens, N_EXPERTS))))
    score = p + bias[None, :]
    if n_group > 1:
        gsz = N_EXPERTS // n_group
        gs = -np.sort(-score.reshape(tokens, n_group, gsz), axis=2)[:, :, :2].sum(axis=2)
        gsel = np.argsort(-gs, axis=1, kind="stable")[:, :topk_group]
        mask = np.zeros((tokens, n_group), bool)
        np.put_along_axis(mask, gsel, True, axis=1)
        score = np.where(np.repeat(mask, gsz, axis=1), score, -np.inf)
    sel = np.argpartition(-score, topk, axis=1)[:, :topk]
    psel = np.take_along_axis(p, sel, axis=1)
    kept = np.take_along_axis(sel, np.argsort(-psel, axis=1)[:, :keep], axis=1)
    return np.bincount(kept.reshape(-1), minlength=N_EXPERTS)


def calibrate_zipf_lambda(target=10.0, keep=2, s=1.2, seed=0x21F, iters=18, n_group=1, topk_group=1):
    """Bisection on lam for hottest / mean = target (simulated routing)."""
    lo, hi = 0.0, 1.0
    for _ in range(iters):
        mid = 0.5 * (lo + hi)
        c = simulate_counts(zipf_bias(mid, s, seed), keep, n_group=n_group, topk_group=topk_group)
        ratio = c.max() / c.mean()
        lo, hi = (mid, hi) if ratio < target else (lo, mid)
    return 0.5 * (lo + hi)
