"""Distribution pin of the rejection-sampling acceptance rule.

The reference has no speculative sampling (deepseek_v4_ds4.c:75-85 rejects
temperature > 0 with more than one draft), so the rule cannot be pinned
against reference outputs.  It is pinned by its defining property instead
(Leviathan et al. 2023, Theorem 1; Chen et al. 2023): whatever the drafts,
the emitted tokens are distributed as if each were sampled from the target,
p_i = softmax(logits_i / T).  For a drafter whose proposal is a point mass
(the planted / greedy drafts here), the rule accepts draft d with probability
p(d) and on rejection samples from p with d removed and renormalised; a
fully accepted round samples a bonus token from the last row.

Checked with Pearson chi-square tests over many Philox counters on a small
vocabulary, for the oracle's restatement (CPU) and for the device kernels
through fc_test_accept (GPU), whose decisions must also equal the oracle's
counter by counter."""
import ctypes

import numpy as np
import pytest
from scipy.stats import chisquare

V = 8
T = 0.7
TRIALS = 20000
P_MIN = 1e-4   # seeded, so deterministic; a correct rule passes with a wide margin


def logits_rows(rows, seed=3):
    rng = np.random.default_rng(seed)
    return (rng.standard_normal((rows, V)) * 1.5).astype(np.float32)


def chi_p(observed, probs):
    """Pearson chi-square p-value of counts against probabilities."""
    probs = np.asarray(probs, dtype=np.float64)
    observed = np.asarray(observed, dtype=np.float64)
    return chisquare(observed, probs / probs.sum() * observed.sum()).pvalue


def softmax_t(x):
    z = np.exp((x.astype(np.float64) - x.max()) / T)
    return z / z.sum()


def oracle_trials(oracle_lib, logits, ids, counter0, trials):
    L = oracle_lib.lib()
    lg = np.ascontiguousarray(logits, dtype=np.float32)
    idp = np.ascontiguousarray(ids, dtype=np.int32)
    commits = np.zeros(trials, dtype=np.int32)
    nxt = np.zeros(trials, dtype=np.int32)
    n = ctypes.c_int()
    for t in range(trials):
        commits[t] = L.orc_accept_sample(lg.ctypes.data_as(ctypes.POINTER(ctypes.c_float)), V,
                                         idp.ctypes.data_as(ctypes.POINTER(ctypes.c_int)),
                                         len(ids) - 1, T, 1, counter0 + t, ctypes.byref(n))
        nxt[t] = n.value
    return commits, nxt


def emitted_tokens(ids, commits, nxt):
    """Per trial, the tokens after ids[0]: accepted drafts, then the sampled
    next token."""
    out = []
    for c, n in zip(commits, nxt):
        out.append(list(ids[1:c]) + [int(n)])
    return out


def check_distribution(logits, ids, commits, nxt):
    k = len(ids) - 1
    toks = emitted_tokens(ids, commits, nxt)
    # position 1 (the first emitted token after ids[0]) ~ p_0
    first = np.bincount([t[0] for t in toks], minlength=V)
    p0 = softmax_t(logits[0])
    assert chi_p(first, p0) > P_MIN
    # accept probability of the first draft = p_0(d_1)
    acc = float(np.mean(commits >= 2))
    assert abs(acc - p0[ids[1]]) < 5 * np.sqrt(p0[ids[1]] * (1 - p0[ids[1]]) / len(toks)) + 1e-3
    # the bonus token of fully accepted rounds ~ p_k
    full = nxt[commits == k + 1]
    if len(full) > 500:
        pk = softmax_t(logits[k])
        assert chi_p(np.bincount(full, minlength=V), pk) > P_MIN
    # a rejection of d_1 resamples from p_0 without d_1
    rej = nxt[commits == 1]
    q = p0.copy()
    q[ids[1]] = 0
    q /= q.sum()
    cnt = np.bincount(rej, minlength=V)
    assert cnt[ids[1]] == 0
    keep = q > 0
    assert chi_p(cnt[keep], q[keep]) > P_MIN


@pytest.mark.parametrize("ids", [[0, 2, 5], [1, 1, 1, 1], [3, 7]])
def test_oracle_sampling_emits_target_distribution(oracle_lib, ids):
    logits = logits_rows(len(ids))
    # make the drafts likely enough that full accepts happen
    for i in range(1, len(ids)):
        logits[i - 1, ids[i]] += 1.0
    commits, nxt = oracle_trials(oracle_lib, logits, ids, 1000, TRIALS)
    check_distribution(logits, ids, commits, nxt)


@pytest.mark.gpu
@pytest.mark.parametrize("ids", [[0, 2, 5], [1, 1, 1, 1], [3, 7]])
def test_device_sampling_emits_target_distribution(fc, oracle_lib, ids):
    logits = logits_rows(len(ids))
    for i in range(1, len(ids)):
        logits[i - 1, ids[i]] += 1.0
    commits, nxt = fc.accept_trials(logits, ids, temperature=T, seed=1, counter=1000, trials=TRIALS)
    check_distribution(logits, ids, commits, nxt)
    oc, on = oracle_trials(oracle_lib, logits, ids, 1000, 2000)
    assert np.array_equal(commits[:2000], oc) and np.array_equal(nxt[:2000], on)


@pytest.mark.gpu
def test_device_greedy_acceptance_rule(fc):
    logits = logits_rows(4)
    tops = logits.argmax(axis=1)
    ids = [9 % V, int(tops[0]), int(tops[1]), (int(tops[2]) + 1) % V]
    commits, nxt = fc.accept_trials(logits, ids, mode=fc.ACCEPT_GREEDY, trials=3)
    assert list(commits) == [3, 3, 3] and list(nxt) == [int(tops[2])] * 3
