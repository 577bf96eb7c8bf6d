"""The benchmark configurations end to end on the GPU, each against the CPU oracle of the
reference forward (``oracle/forward_ref.py``, ``MlxBackend::forward``,
runtime/crates/laya-mlx/src/lib.rs:1833-1863) or a PyTorch fp32 reference:

  cfg1  1 row x 128 tokens, one noul question                        -> oracle parity
  cfg2  1 row x 512 tokens with 10 questions (30 markers), and the same questions as 10 rows
        (the state segment plus one question segment each)            -> oracle parity
  cfg3  64 rows of U[64, 512] tokens, 3 questions each, one varlen batch -> every row against the
        oracle run on that row alone
  cfg4  the encoder GEMM sweep: M in {128, 512, 2048, 8192, 32768} x (Wqkv + RoPE, Wi + GeGLU,
        Wo2 K = 2624) with the epilogue each runs with in the forward  -> PyTorch fp32
  cfg5  one GPU's shard of the serving run (1024 lognormal requests, varlen batches of <= 16384
        tokens): too large for the oracle, so size-independent properties over the whole shard
        (finite outputs, masked slots exactly -1e4, bit-identical on a second run) and a spread
        sample of requests against the oracle.

Tolerances as in test_gpu_forward.py: per-question probabilities within 1e-2, hidden states within
2e-2 relative, choice argmax equal where the oracle's margin exceeds the logit error.
"""
import numpy as np
import pytest
import torch

from sys1rust_b200.batch import EncodedItem, Varlen, collate_to

pytestmark = pytest.mark.gpu

HIDDEN_REL = 2e-2
PROB_ABS = 1e-2


@pytest.fixture(scope="module")
def large():
    from conftest import get_backend
    from oracle.forward_ref import OracleModel
    cfg, w, be = get_backend("large:0")
    return cfg, w, be, OracleModel(cfg, w.tensors)


def _check_row(got_logits, got_pooled, got_hidden, item, om, cfg):
    """One request's outputs against the oracle run on that request alone."""
    lo, po, ho = om.forward(collate_to([item], cfg.encoder.pad_token_id))
    k = len(item.markers)
    L = len(item.ids)
    hid = np.asarray(got_hidden).reshape(L, -1)
    rel = np.linalg.norm(hid - ho[0, :L]) / np.linalg.norm(ho[0, :L])
    assert rel < HIDDEN_REL, f"hidden rel err {rel}"
    g = np.asarray(got_logits[:k], np.float64)
    o = np.asarray(lo[:k], np.float64)
    err = np.abs(g - o).max() if k else 0.0
    # option probabilities over the row's markers (one row = one typed question group, as in
    # test_gpu_forward.question_probs)
    pg, pw = np.exp(g - g.max()) if k else g, np.exp(o - o.max()) if k else o
    if k:
        assert np.abs(pg / pg.sum() - pw / pw.sum()).max() < PROB_ABS
    srt = np.sort(o)
    if k >= 2 and srt[-1] - srt[-2] > 2 * err:
        assert np.argmax(g) == np.argmax(o)
    prel = np.linalg.norm(got_pooled - po) / np.linalg.norm(po)
    assert prel < 5e-2, f"pooled rel err {prel}"
    return rel


def _run_varlen(be, items):
    v = Varlen.from_rows(items)
    out = be.forward_varlen(v, hidden=True)
    d = be.hidden
    return v, out.logits.reshape(v.n, v.kmax), out.pooled.reshape(v.n, d), out.hidden.reshape(v.total, d)


def test_cfg1_single_request(cuda_lib, large):
    from sys1rust_b200.workloads import cfg1
    cfg, w, be, om = large
    items = cfg1()
    v, lg, pl, hd = _run_varlen(be, items)
    _check_row(lg[0], pl[0], hd, items[0], om, cfg)


def test_cfg2_one_row_and_ten_rows(cuda_lib, large):
    from sys1rust_b200.workloads import cfg2
    cfg, w, be, om = large
    row = cfg2()[0]
    assert len(row.ids) == 512 and len(row.markers) == 30
    v, lg, pl, hd = _run_varlen(be, [row])
    _check_row(lg[0], pl[0], hd, row, om, cfg)
    # the reference's semantics: one row per question, the 462-token state plus that question's
    # 5-token segment, one marker per option at the start of the segment, the row typed by its
    # question (4 choice x 3 options, 3 score x 4, 3 noul x 2)
    from sys1rust_b200.workloads import LABELS
    state = list(row.ids[:462])
    rows = []
    for q, t in enumerate([0] * 4 + [1] * 3 + [2] * 3):
        seg = list(row.ids[462 + 5 * q: 467 + 5 * q])
        rows.append(EncodedItem(state + seg, [462 + j for j in range(LABELS[t])], t))
    v, lg, pl, hd = _run_varlen(be, rows)
    off = np.concatenate([[0], np.cumsum([len(r.ids) for r in rows])])
    for i, r in enumerate(rows):
        _check_row(lg[i], pl[i], hd[off[i]:off[i + 1]], r, om, cfg)


def test_cfg3_throughput_batch(cuda_lib, large):
    from sys1rust_b200.workloads import cfg3
    cfg, w, be, om = large
    items = cfg3()
    assert len(items) == 64
    v, lg, pl, hd = _run_varlen(be, items)
    off = np.asarray(v.cu_seqlens)
    rels = [_check_row(lg[i], pl[i], hd[off[i]:off[i + 1]], it, om, cfg) for i, it in enumerate(items)]
    print(f"cfg3: T = {v.total}, worst hidden rel err {max(rels):.4g}")


def _rand(shape, seed):
    g = torch.Generator(device="cpu").manual_seed(seed)
    return torch.randn(*shape, generator=g).to(torch.bfloat16).cuda()


def _rel(out, ref):
    return (out.float() - ref).abs().max().item() / ref.abs().max().item()


@pytest.mark.parametrize("M", [128, 512, 2048, 8192, 32768])
def test_cfg4_gemm_sweep(cuda_lib, M):
    from sys1rust_b200.backend import EPI_GEGLU, EPI_RESID, EPI_ROPE, gemm, interleave_wi
    from test_gpu_kernels import _rope_ref
    d, I = 1024, 2624
    # Wqkv + split/RoPE (positions 0..M-1 of one row, theta 160000)
    a, b = _rand((M, d), 41), _rand((3 * d, d), 42)
    pos = torch.arange(M, dtype=torch.int32, device="cuda") % 8192
    out = torch.empty(M, 3 * d, dtype=torch.bfloat16, device="cuda")
    gemm(EPI_ROPE, a.data_ptr(), b.data_ptr(), out.data_ptr(), M, 3 * d, d, pos_ptr=pos.data_ptr(),
         rope_theta=160000.0, rope_cols=2 * d)
    torch.cuda.synchronize()
    acc = a.float() @ b.float().t()
    assert _rel(out, torch.cat([_rope_ref(acc[:, :2 * d], pos, 160000.0), acc[:, 2 * d:]], 1)) < 1e-2
    del acc, out
    # Wi + GeGLU
    wi = _rand((2 * I, d), 43)
    wil = torch.from_numpy(interleave_wi(wi.cpu().view(torch.int16).numpy(), I)).view(torch.bfloat16).cuda()
    out = torch.empty(M, I, dtype=torch.bfloat16, device="cuda")
    gemm(EPI_GEGLU, a.data_ptr(), wil.data_ptr(), out.data_ptr(), M, wil.shape[0], d, out_cols=I)
    torch.cuda.synchronize()
    y = a.float() @ wi.float().t()
    assert _rel(out, torch.nn.functional.gelu(y[:, :I]) * y[:, I:]) < 1e-2
    del y, out
    # Wo2 (K = 2624) adding into the fp32 residual stream
    a2, b2 = _rand((M, I), 44), _rand((d, I), 45)
    h0 = torch.randn(M, d, generator=torch.Generator().manual_seed(46)).float().cuda()
    h = h0.clone()
    gemm(EPI_RESID, a2.data_ptr(), b2.data_ptr(), h.data_ptr(), M, d, I)
    torch.cuda.synchronize()
    assert _rel(h, h0 + a2.float() @ b2.float().t()) < 1e-4


def test_cfg5_shard_properties_and_sample(cuda_lib, large):
    from sys1rust_b200.workloads import cfg5_requests, pack_batches, shard_lpt
    cfg, w, be, om = large
    shard = shard_lpt(cfg5_requests(), 8)[0]  # rank 0 of the 8-GPU run
    batches = pack_batches(shard, 16384)
    assert all(b.total <= 16384 for b in batches)
    runs = []
    for _ in range(2):
        runs.append([be.forward_varlen(b) for b in batches])
    for b, o1, o2 in zip(batches, *runs):
        assert np.array_equal(o1.logits, o2.logits) and np.array_equal(o1.pooled, o2.pooled)
        assert np.isfinite(o1.logits).all() and np.isfinite(o1.pooled).all()
        lg = o1.logits.reshape(b.n, b.kmax)
        for r in range(b.n):
            assert np.all(lg[r, int(b.marker_count[r]):] == np.float32(-1e4))
    # a spread sample against the oracle: the shortest, the longest and a few in between
    flat = [(bi, r) for bi, b in enumerate(batches) for r in range(b.n)]
    lens = np.array([int(batches[bi].cu_seqlens[r + 1] - batches[bi].cu_seqlens[r]) for bi, r in flat])
    order = np.argsort(lens)
    pick = sorted(set([order[0], order[-1]] + [order[int(q * (len(order) - 1))] for q in (0.25, 0.5, 0.75)]))
    for p in pick:
        bi, r = flat[p]
        b = batches[bi]
        s, e = int(b.cu_seqlens[r]), int(b.cu_seqlens[r + 1])
        k = int(b.marker_count[r])
        item = EncodedItem([int(x) for x in b.ids[s:e]], [int(x) for x in b.marker_pos[r * b.kmax: r * b.kmax + k]],
                           int(b.qtype[r]))
        out = be.forward_varlen(b, hidden=True)
        hd = out.hidden.reshape(b.total, -1)[s:e]
        _check_row(out.logits.reshape(b.n, b.kmax)[r], out.pooled.reshape(b.n, -1)[r], hd, item, om, cfg)
