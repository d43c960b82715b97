"""Batched multi-sequence verify (fc_session_create_batch / _verify_batch):
several sequences over one paged latent cache with a shared prefix, packed
floor(8 / rows) sequences per device pass.

  - every sequence's commit, next token and verify-row logits equal those of
    the same verify in a one-sequence batch session, bit for bit (rows are
    independent in every kernel, and a query tile never mixes sequences);
  - against per-sequence oracle sessions: the same commits and next tokens
    (greedy), with prefix positions shared and private tails of different
    lengths and seeds, so a wrong page-table entry reads other KV;
  - rejection sampling with per-sequence Philox counters;
  - per-sequence positions and rollback; invalid shapes are refused."""
import numpy as np
import pytest

from floyd_b200 import ACCEPT_GREEDY, ACCEPT_SAMPLE, CONFIGS, scaled
from test_gpu_attention_tc import C4_TC
from test_gpu_verify import C1, C4_SMALL, MARGIN, pair

pytestmark = pytest.mark.gpu

PREFIX = 64
PREFIX_SEED = 7
CTX = 320
TAILS = [150, 201, 266]        # context length of each sequence


def _seed_batch(bs, n):
    bs.seed(0, 0, PREFIX, PREFIX_SEED)
    for q in range(n):
        bs.seed(q, PREFIX, TAILS[q], 100 + q)


def _ids(cfg, q, rows):
    rng = np.random.default_rng(50 + q)
    return rng.integers(0, cfg["vocab_size"], size=rows).tolist()


def _single(cfg, name, q, rows, accept=None):
    import floyd_b200
    gm, _ = pair(cfg, name)
    s = floyd_b200.BatchSession(gm, CTX, 1, rows, PREFIX)
    s.seed(0, 0, PREFIX, PREFIX_SEED)
    s.seed(0, PREFIX, TAILS[q], 100 + q)
    n, nxt = s.verify_batch([_ids(cfg, q, rows)], None if accept is None else [accept])
    return n[0], nxt[0], s.row_logits(rows), s.position_of(0)


CASES = [("c1", C1), ("c4s", C4_SMALL), ("c4tc", C4_TC)]


@pytest.mark.parametrize("name,cfg", CASES)
def test_batch_equals_one_sequence_sessions(name, cfg):
    import floyd_b200
    gm, _ = pair(cfg, name)
    rows, n = 4, 3
    bs = floyd_b200.BatchSession(gm, CTX, n, rows, PREFIX)
    _seed_batch(bs, n)
    ids = [_ids(cfg, q, rows) for q in range(n)]
    got_n, got_next = bs.verify_batch(ids)
    last = bs.row_logits(rows)          # the last pass holds only sequence 2
    for q in range(n):
        en, enx, elog, epos = _single(cfg, name, q, rows)
        assert (got_n[q], got_next[q]) == (en, enx), f"sequence {q}"
        assert bs.position_of(q) == epos == TAILS[q] + en
        if q == n - 1:
            assert np.array_equal(last, elog)


@pytest.mark.parametrize("name,cfg", CASES)
def test_batch_matches_oracle_sequences(name, cfg):
    import floyd_b200
    from oracle import oracle
    gm, om = pair(cfg, name)
    rows, n = 4, 3
    bs = floyd_b200.BatchSession(gm, CTX, n, rows, PREFIX)
    _seed_batch(bs, n)
    ids = [_ids(cfg, q, rows) for q in range(n)]
    got_n, got_next = bs.verify_batch(ids)
    for q in range(n):
        os_ = oracle.OracleSession(om, CTX, kv_fp16=True)
        os_.seed_range(0, PREFIX, PREFIX_SEED)
        os_.seed_range(PREFIX, TAILS[q], 100 + q)
        emitted, nxt, logits, _ = os_.verify(ids[q])
        if (len(emitted), nxt) != (got_n[q], got_next[q]):
            # the only allowed difference: a near-tie top-1 on the deciding row
            r = min(len(emitted), got_n[q]) - 1
            part = np.partition(logits[r], -2)
            assert part[-1] - part[-2] < MARGIN, f"sequence {q}: {(len(emitted), nxt)} vs {(got_n[q], got_next[q])}"


def test_batch_sampling_equals_one_sequence_sessions():
    import floyd_b200
    cfg, name = C4_SMALL, "c4s"
    gm, _ = pair(cfg, name)
    rows, n = 4, 3
    acc = [(ACCEPT_SAMPLE, 0.7, 1, 10 + q) for q in range(n)]
    bs = floyd_b200.BatchSession(gm, CTX, n, rows, PREFIX)
    _seed_batch(bs, n)
    got_n, got_next = bs.verify_batch([_ids(cfg, q, rows) for q in range(n)], acc)
    for q in range(n):
        en, enx, _, _ = _single(cfg, name, q, rows, acc[q])
        assert (got_n[q], got_next[q]) == (en, enx), f"sequence {q}"


def test_batch_positions_rollback_and_steps():
    """Several steps: each sequence advances by its own commit; a rollback of
    one sequence leaves the others alone and its next verify re-writes the
    rolled-back positions."""
    import floyd_b200
    cfg, name = C1, "c1"
    gm, _ = pair(cfg, name)
    rows, n = 2, 5          # 4 sequences per pass, two passes
    bs = floyd_b200.BatchSession(gm, CTX, n, rows, PREFIX)
    bs.seed(0, 0, PREFIX, PREFIX_SEED)
    for q in range(n):
        bs.seed(q, PREFIX, 100 + 10 * q, 100 + q)
    pos = [bs.position_of(q) for q in range(n)]
    assert pos == [100 + 10 * q for q in range(n)]
    nxt = [1] * n
    for step in range(3):
        ids = [[nxt[q], (nxt[q] + 1) % cfg["vocab_size"]] for q in range(n)]
        got_n, nxt = bs.verify_batch(ids)
        pos = [p + c for p, c in zip(pos, got_n)]
        assert [bs.position_of(q) for q in range(n)] == pos
    bs.rollback_seq(2, pos[2] - 1)
    assert bs.position_of(2) == pos[2] - 1 and bs.position_of(1) == pos[1]


def test_batch_refuses_invalid_shapes():
    import floyd_b200
    gm, _ = pair(C1, "c1")
    with pytest.raises(floyd_b200.FloydError):
        floyd_b200.BatchSession(gm, CTX, 2, 3, PREFIX)        # 3 rows x 16 heads: tiles would mix sequences
    with pytest.raises(floyd_b200.FloydError):
        floyd_b200.BatchSession(gm, CTX, 2, 4, 100)           # prefix not a whole number of pages
    bs = floyd_b200.BatchSession(gm, CTX, 2, 4, PREFIX)
    with pytest.raises(floyd_b200.FloydError):
        bs.decode(1)                                          # single-sequence calls are refused
    with pytest.raises(floyd_b200.FloydError):
        bs.verify_batch([[1, 2, 3, 4], [5, 6, 7, 8]])          # sequences without context
    bs.seed(0, 0, 32, 7)
    bs.seed(1, 0, 200, 8)
    with pytest.raises(floyd_b200.FloydError):
        bs.verify_batch([[1, 2, 3, 4], [5, 6, 7, 8]])          # sequence 0 would write into the shared pages
    bs.seed(0, 32, 100, 9)
    bs.verify_batch([[1, 2, 3, 4], [5, 6, 7, 8]])


def test_concurrent_passes_equal_sequential_passes(monkeypatch):
    """The passes of a batch step run concurrently on lanes (own stream and
    workspace over the shared cache); the results and the last pass's logits
    equal those of the same steps run one pass at a time, bit for bit."""
    import floyd_b200
    name, cfg = CASES[2]
    gm, _ = pair(cfg, name)
    rows, n = 4, 3
    out = []
    for lanes in ("1", "4"):
        monkeypatch.setenv("FLOYD_BATCH_LANES", lanes)
        bs = floyd_b200.BatchSession(gm, CTX, n, rows, PREFIX)
        _seed_batch(bs, n)
        steps = []
        for step in range(3):
            ids = [_ids(cfg, 10 * step + q, rows) for q in range(n)]
            got_n, got_next = bs.verify_batch(ids)
            steps.append((list(got_n), list(got_next), [bs.position_of(q) for q in range(n)],
                          bs.row_logits(rows).copy()))
        out.append(steps)
    for a, b in zip(*out):
        assert a[:3] == b[:3]
        assert np.array_equal(a[3], b[3])
