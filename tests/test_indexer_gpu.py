"""GPU parity of the indexer top-k (ws_indexer_topk) against the reference's
golden output (indexer_topk_cpu, kernel/cpu_attn_ds4_ext/csa_attn.cpp:1658-1736)
and the float64 oracle.

fp32 inputs are scored in the reference's own order of operations, so the
scores equal the oracle's fp32 restatement bit for bit and the ids equal the
reference's (test_golden_large: same sets, same order up to runs of exactly
equal scores, which the reference's partial_sort leaves unordered).  bf16
inputs (tensor-core scoring, no reference counterpart) are checked up to
near-ties at the k-th score: every selected entry scores at least s_k - eps
and every other entry at most s_k + eps (eps = 1e-5 of the score scale);
exact ties are ordered by id.
"""
import numpy as np
import pytest
import torch

import oracle
import scope_b200
import scope_b200.csa_attn   # the submodule is imported on first use, not by the package

pytestmark = pytest.mark.gpu
DEV = "cuda:0"


@pytest.fixture(scope="module")
def csa():
    return scope_b200.build_csa_attn()


def check_selection(ids, scores_ref, k, order="score", our_scores=None):
    bs = scores_ref.shape[0]
    for b in range(bs):
        s = scores_ref[b]
        sel = ids[b]
        assert len(set(sel.tolist())) == len(sel) == min(k, s.shape[0])
        eps = 1e-5 * (np.abs(s).max() + 1.0)
        t = np.sort(s)[::-1][len(sel) - 1]
        mask = np.zeros(s.shape[0], bool)
        mask[sel] = True
        assert s[mask].min() >= t - eps
        if (~mask).any():
            assert s[~mask].max() <= t + eps
        if order == "id":
            assert np.all(np.diff(sel) > 0)
        elif our_scores is not None:
            o = our_scores[b][sel]
            assert np.all(np.diff(o) <= 0)
            ties = np.diff(o) == 0
            assert np.all(np.diff(sel)[ties] > 0)


def rand_case(bs, nH, hd, nc, seed, dtype=torch.float32):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(bs, nH, hd, generator=g)
    kv = torch.randn(bs, nc, hd, generator=g)
    w = torch.rand(bs, nH, generator=g) - 0.3     # some negative weights, as a learned projection gives
    if dtype == torch.bfloat16:
        q, kv = q.bfloat16(), kv.bfloat16()
    return q, kv, w


def oracle_scores(q, kv, w, k):
    ids, sc = oracle.indexer_topk(q.float().numpy(), kv.float().numpy(), w.numpy(), k)
    return ids, sc


def test_golden(csa, golden):
    g = golden("indexer_topk")
    k = int(g["k"])
    ids = csa.indexer_topk_cpu(torch.from_numpy(g["q_idx"]).to(DEV), torch.from_numpy(g["kv_idx"]).to(DEV),
                               torch.from_numpy(g["weights"]).to(DEV), k)
    assert ids.dtype == torch.int32 and tuple(ids.shape) == (g["ids"].shape[0], k)
    _, sc = oracle.indexer_topk(g["q_idx"], g["kv_idx"], g["weights"], k)
    check_selection(ids.cpu().numpy(), sc, k)
    for b in range(ids.shape[0]):     # the reference's own set
        assert set(ids[b].tolist()) == set(g["ids"][b].tolist())


@pytest.mark.parametrize("bs,nH,hd,nc,k", [(1, 1, 16, 10, 3), (2, 4, 64, 200, 16), (3, 8, 128, 5000, 100),
                                           (2, 64, 128, 20000, 2048), (1, 16, 256, 4096, 4096),
                                           (2, 5, 48, 777, 777), (1, 3, 32, 100, 500), (1, 8, 64, 20000, 3000),
                                           (2, 4, 32, 9001, 700), (5, 2, 64, 33333, 2048)])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_random(csa, bs, nH, hd, nc, k, dtype):
    q, kv, w = rand_case(bs, nH, hd, nc, seed=bs * 7919 + nc + k, dtype=dtype)
    ids, our = scope_b200.csa_attn.indexer_topk(q.to(DEV), kv.to(DEV), w.to(DEV), k, return_scores=True)
    _, sc = oracle_scores(q, kv, w, k)
    our = our.cpu().numpy()
    assert np.abs(our - sc).max() <= 1e-5 * (np.abs(sc).max() + 1.0)
    check_selection(ids.cpu().numpy(), sc, k, our_scores=our)
    ids_id = scope_b200.csa_attn.indexer_topk(q.to(DEV), kv.to(DEV), w.to(DEV), k, order="id")
    check_selection(ids_id.cpu().numpy(), sc, k, order="id")
    assert all(set(a.tolist()) == set(b.tolist()) for a, b in zip(ids.cpu(), ids_id.cpu()))


def test_exact_ties_take_lower_ids_first():
    g = torch.Generator().manual_seed(3)
    nc, hd = 1000, 32
    base = torch.randn(10, hd, generator=g)
    kv = base[torch.randint(0, 10, (nc,), generator=g)][None]       # only 10 distinct rows: many exact ties
    q = torch.randn(1, 2, hd, generator=g)
    w = torch.ones(1, 2)
    ids, our = scope_b200.csa_attn.indexer_topk(q.to(DEV), kv.contiguous().to(DEV), w.to(DEV), 150,
                                                return_scores=True)
    ids, our = ids.cpu().numpy()[0], our.cpu().numpy()[0]
    order = sorted(range(nc), key=lambda j: (-our[j], j))[:150]     # descending score, then ascending id
    assert ids.tolist() == order


@pytest.mark.parametrize("nc,distinct,k", [(30000, 10, 150), (20000, 3000, 2048), (50000, 1, 7)])
def test_ties_beyond_the_candidate_buffer(nc, distinct, k):
    """More scores than the shared-memory candidate buffer holds, with heavy ties: the sampled
    threshold then passes too many keys (or exactly-equal ones straddle it) and the select runs over
    all scores; ties still go to the lowest ids first."""
    g = torch.Generator().manual_seed(nc + distinct)
    base = torch.randn(distinct, 32, generator=g)
    kv = base[torch.randint(0, distinct, (nc,), generator=g)][None].contiguous()
    q = torch.randn(1, 2, 32, generator=g)
    w = torch.ones(1, 2)
    ids, our = scope_b200.csa_attn.indexer_topk(q.to(DEV), kv.to(DEV), w.to(DEV), k, return_scores=True)
    ids, our = ids.cpu().numpy()[0], our.cpu().numpy()[0]
    order = np.lexsort((np.arange(nc), -our))[:k]     # descending score, then ascending id
    assert ids.tolist() == order.tolist()
    ids_id = scope_b200.csa_attn.indexer_topk(q.to(DEV), kv.to(DEV), w.to(DEV), k, order="id").cpu().numpy()[0]
    assert ids_id.tolist() == sorted(order.tolist())


def _exact_order(scores, k):
    return np.lexsort((np.arange(scores.shape[0]), -scores))[:k]     # descending score, then ascending id


@pytest.mark.parametrize("k", [500, 2048])
def test_one_cta_per_sequence_without_workspace(k):
    """Scores returned to the caller and no workspace: the select runs one CTA per sequence (sampled
    threshold, candidates in shared memory) instead of spreading the candidate pass."""
    from scope_b200 import _lib
    bs, nH, hd, nc = 3, 8, 64, 30000
    q, kv, w = rand_case(bs, nH, hd, nc, seed=k)
    q, kv, w = q.to(DEV), kv.to(DEV), w.to(DEV)
    L = _lib.lib()
    for order in (_lib.WS_TOPK_BY_SCORE, _lib.WS_TOPK_BY_ID):
        ids = torch.empty(bs, k, dtype=torch.int32, device=DEV)
        sc = torch.empty(bs, nc, dtype=torch.float32, device=DEV)
        rc = L.ws_indexer_topk(_lib.ptr(q), _lib.ptr(kv), _lib.WS_DTYPE_F32, _lib.ptr(w), bs, nH, hd, nc, k, order,
                               _lib.ptr(ids), _lib.ptr(sc), None, 0, _lib.stream_ptr(torch.device(DEV)))
        _lib.check(rc, "ws_indexer_topk")
        ids, sc = ids.cpu().numpy(), sc.cpu().numpy()
        for b in range(bs):
            want = _exact_order(sc[b], k)
            assert ids[b].tolist() == (want.tolist() if order == _lib.WS_TOPK_BY_SCORE else sorted(want.tolist()))


def test_many_sequences_one_cta_each():
    """More sequences than half the SMs: one select CTA per sequence even with a workspace."""
    bs, nH, hd, nc, k = 80, 2, 16, 9000, 300
    q, kv, w = rand_case(bs, nH, hd, nc, seed=80)
    ids, our = scope_b200.csa_attn.indexer_topk(q.to(DEV), kv.to(DEV), w.to(DEV), k, return_scores=True)
    ids, our = ids.cpu().numpy(), our.cpu().numpy()
    for b in range(bs):
        assert ids[b].tolist() == _exact_order(our[b], k).tolist()
    _, sc = oracle_scores(q, kv, w, k)
    assert np.abs(our - sc).max() <= 1e-5 * (np.abs(sc).max() + 1.0)


@pytest.mark.parametrize("order", ["score", "id"])
def test_outlier_score(order):
    """One entry scores ~10^4 times the rest: the equal-width buckets over the candidates' range then
    put almost every candidate into a few buckets and the select falls back to radix passes."""
    bs, nH, hd, nc, k = 2, 4, 32, 20000, 2048
    q, kv, w = rand_case(bs, nH, hd, nc, seed=5)
    w = w.abs() + 0.1
    kv[:, 77] = 1e4 * q[:, 0]     # head 0 scores 1e4 |q_0|^2 there
    ids, our = scope_b200.csa_attn.indexer_topk(q.to(DEV), kv.to(DEV), w.to(DEV), k, order=order,
                                                return_scores=True)
    ids, our = ids.cpu().numpy(), our.cpu().numpy()
    for b in range(bs):
        want = _exact_order(our[b], k).tolist()
        assert ids[b].tolist() == (want if order == "score" else sorted(want))


def test_ds4_size():
    """A DeepSeek-V4-like indexer shape: 64 index heads x 128 dims over 65536
    compressed entries, top-2048, two sequences against the oracle."""
    q, kv, w = rand_case(2, 64, 128, 65536, seed=11)
    ids = scope_b200.csa_attn.indexer_topk(q.to(DEV), kv.to(DEV), w.to(DEV), 2048)
    _, sc = oracle_scores(q, kv, w, 2048)
    check_selection(ids.cpu().numpy(), sc, 2048)


def _large_inputs(golden, i):
    g = golden("indexer_topk_large")
    seed, bs, nH, hd, nc, k = (int(x) for x in g[f"c{i}_shape"])
    rng = np.random.default_rng(seed)     # the generator tests/golden/make_golden.py drew them from
    q = rng.standard_normal((bs, nH, hd), dtype=np.float32)
    kv = rng.standard_normal((bs, nc, hd), dtype=np.float32)
    w = rng.random((bs, nH), dtype=np.float32)
    chk = np.array([q.astype(np.float64).sum(), kv.astype(np.float64).sum(), w.astype(np.float64).sum()])
    assert np.array_equal(chk, g[f"c{i}_checksum"]), "numpy's generator no longer reproduces the fixture inputs"
    return q, kv, w, k, g[f"c{i}_ids"]


@pytest.mark.parametrize("i", [0, 1])
def test_golden_large(csa, golden, i):
    """indexer_topk_cpu at nc >= 20000, k = 2048 against the reference's own
    ids: identical sets and identical order up to runs of exactly equal fp32
    scores; the scores themselves equal the fp32 restatement bit for bit."""
    q, kv, w, k, ref = _large_inputs(golden, i)
    ids, scores = csa.indexer_topk(torch.from_numpy(q).to(DEV), torch.from_numpy(kv).to(DEV),
                                   torch.from_numpy(w).to(DEV), k, return_scores=True)
    ids2 = csa.indexer_topk_cpu(torch.from_numpy(q).to(DEV), torch.from_numpy(kv).to(DEV),
                                torch.from_numpy(w).to(DEV), k)
    torch.cuda.synchronize()
    sc = scores.cpu().numpy()
    want = oracle.indexer_scores_f32(q, kv, w, contract=False)
    assert np.array_equal(sc.view(np.uint32), want.view(np.uint32)), int((sc != want).sum())
    agree = oracle.topk_agreement(ids.cpu().numpy(), ref, want)
    assert agree["set_diff"] == 0 and agree["order_diff"] == 0, agree
    assert np.array_equal(ids2.cpu().numpy(), ids.cpu().numpy())
