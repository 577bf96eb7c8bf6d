"""Kernel-level parity on the GPU: each sm_100a kernel against a plain PyTorch fp32 reference of
the same op, through the C ABI (``s1c_gemm``, ``s1c_attention``).

Tolerances: outputs stored as bf16 carry a relative rounding error of 2^-9; the bound used is
``max|out - ref| <= 1e-2 * max|ref|`` (fp32 outputs: 1e-4 relative to the accumulation).
"""
import math

import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu


def _rel_err(out, ref):
    return (out.float() - ref.float()).abs().max().item() / max(ref.float().abs().max().item(), 1e-30)


def _rand(shape, seed, scale=1.0):
    g = torch.Generator(device="cpu").manual_seed(seed)
    return (torch.randn(*shape, generator=g) * scale).to(torch.bfloat16).cuda()


# one-CTA 128x256 tiles, two-CTA 256x256 tiles, workspace split-K, cluster split-K, one-CTA 128x128
VARIANTS = [1, 2, 3, 4, 5]


@pytest.mark.parametrize("variant", VARIANTS)
@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (300, 768, 1024), (1024, 3072, 1024), (77, 1024, 2624),
                                   (513, 256, 4096)])
def test_gemm_store_matches_torch(cuda_lib, M, N, K, variant):
    from sys1rust_b200.backend import EPI_STORE, gemm
    a, b = _rand((M, K), 1), _rand((N, K), 2)
    out = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
    gemm(EPI_STORE, a.data_ptr(), b.data_ptr(), out.data_ptr(), M, N, K, variant=variant)
    torch.cuda.synchronize()
    ref = a.float() @ b.float().t()
    assert _rel_err(out, ref) < 1e-2


@pytest.mark.parametrize("variant", VARIANTS)
@pytest.mark.parametrize("act", [0, 1, 2])
def test_gemm_bias_activation_fp32_out(cuda_lib, act, variant):
    from sys1rust_b200.backend import EPI_STORE, gemm
    M, N, K = 200, 512, 1024
    a, b = _rand((M, K), 3), _rand((N, K), 4)
    bias = torch.randn(N, generator=torch.Generator().manual_seed(5)).float().cuda()
    out = torch.empty(M, N, dtype=torch.float32, device="cuda")
    gemm(EPI_STORE, a.data_ptr(), b.data_ptr(), out.data_ptr(), M, N, K, bias_ptr=bias.data_ptr(), act=act, out_f32=1,
         variant=variant)
    torch.cuda.synchronize()
    ref = a.float() @ b.float().t() + bias
    ref = [ref, torch.relu(ref), torch.nn.functional.gelu(ref)][act]
    assert _rel_err(out, ref) < 1e-4


@pytest.mark.parametrize("variant", VARIANTS)
def test_gemm_residual_in_place(cuda_lib, variant):
    from sys1rust_b200.backend import EPI_RESID, gemm
    M, N, K = 333, 1024, 2624
    a, b = _rand((M, K), 6), _rand((N, K), 7)
    h = torch.randn(M, N, generator=torch.Generator().manual_seed(8)).float().cuda()
    ref = h + a.float() @ b.float().t()
    gemm(EPI_RESID, a.data_ptr(), b.data_ptr(), h.data_ptr(), M, N, K, variant=variant)
    torch.cuda.synchronize()
    assert _rel_err(h, ref) < 1e-4


@pytest.mark.parametrize("variant", VARIANTS)
def test_gemm_residual_f16_in_place(cuda_lib, variant):
    """The encoder's residual stream is f16: out = f16(h + A B^T + bias), the add done by the TMA
    reduction (one-CTA / two-CTA tiles: f16(h + f16(acc))) or once in fp32 (split-K paths). Bound:
    two f16 roundings, 2^-10 relative to the largest output."""
    from sys1rust_b200.backend import EPI_RESID16, gemm
    M, N, K = 333, 1024, 2624
    a, b = _rand((M, K), 6), _rand((N, K), 7)
    bias = torch.randn(N, generator=torch.Generator().manual_seed(9)).float().cuda()
    h = torch.randn(M, N, generator=torch.Generator().manual_seed(8)).half().cuda()
    ref = h.float() + a.float() @ b.float().t() + bias
    gemm(EPI_RESID16, a.data_ptr(), b.data_ptr(), h.data_ptr(), M, N, K, bias_ptr=bias.data_ptr(), variant=variant)
    torch.cuda.synchronize()
    assert _rel_err(h, ref) < 2e-3


@pytest.mark.parametrize("M", [1, 17, 128, 200, 256])
@pytest.mark.parametrize("N,K", [(1024, 64), (1024, 128), (1024, 1024), (3072, 1024), (1024, 2624), (256, 4096)])
def test_cluster_split_k_shapes(cuda_lib, M, N, K):
    """Cluster split-K over cluster sizes 1..4 (K of 1, 2, 16, 41 and 64 blocks) and both tile
    widths; the result is bit-identical from one call to the next (partials summed in rank order)."""
    from sys1rust_b200.backend import EPI_RESID, EPI_STORE, gemm
    a, b = _rand((M, K), 31), _rand((N, K), 32)
    out = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
    gemm(EPI_STORE, a.data_ptr(), b.data_ptr(), out.data_ptr(), M, N, K, variant=4)
    torch.cuda.synchronize()
    assert _rel_err(out, a.float() @ b.float().t()) < 1e-2
    h0 = torch.randn(M, N, generator=torch.Generator().manual_seed(33)).float().cuda()
    outs = []
    for _ in range(2):
        h = h0.clone()
        gemm(EPI_RESID, a.data_ptr(), b.data_ptr(), h.data_ptr(), M, N, K, variant=4)
        torch.cuda.synchronize()
        outs.append(h)
    assert _rel_err(outs[0], h0 + a.float() @ b.float().t()) < 1e-4
    assert torch.equal(outs[0], outs[1])
    from sys1rust_b200.backend import EPI_RESID16
    h16 = h0.half()
    outs = []
    for _ in range(2):
        h = h16.clone()
        gemm(EPI_RESID16, a.data_ptr(), b.data_ptr(), h.data_ptr(), M, N, K, variant=4)
        torch.cuda.synchronize()
        outs.append(h)
    assert _rel_err(outs[0], h16.float() + a.float() @ b.float().t()) < 2e-3
    assert torch.equal(outs[0], outs[1])


def _rope_ref(x, pos, theta):
    """Rotate-half RoPE per 64-wide head of x [M, C] at positions pos [M] (split_rope.metal:46-76)."""
    M, Cc = x.shape
    half = 32
    lbase = torch.log2(torch.tensor(theta, dtype=torch.float32))
    inv = torch.exp2(-(torch.arange(half, dtype=torch.float32) / half) * lbase)
    ang = pos.float().cpu()[:, None] * inv[None, :]
    c, s = torch.cos(ang).cuda(), torch.sin(ang).cuda()
    xh = x.view(M, Cc // 64, 64)
    x1, x2 = xh[..., :half], xh[..., half:]
    return torch.cat([x1 * c[:, None] - x2 * s[:, None], x1 * s[:, None] + x2 * c[:, None]], -1).view(M, Cc)


@pytest.mark.parametrize("variant", VARIANTS)
@pytest.mark.parametrize("theta", [160000.0, 10000.0])
def test_gemm_rope_epilogue(cuda_lib, theta, variant):
    from sys1rust_b200.backend import EPI_ROPE, gemm
    d = 1024
    M, N, K = 700, 3 * d, d
    a, b = _rand((M, K), 9), _rand((N, K), 10)
    pos = torch.from_numpy(np.concatenate([np.arange(500), np.arange(200)]).astype(np.int32)).cuda()
    out = torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
    gemm(EPI_ROPE, a.data_ptr(), b.data_ptr(), out.data_ptr(), M, N, K, pos_ptr=pos.data_ptr(), rope_theta=theta,
         rope_cols=2 * d, variant=variant)
    torch.cuda.synchronize()
    acc = a.float() @ b.float().t()
    ref = torch.cat([_rope_ref(acc[:, :2 * d], pos, theta), acc[:, 2 * d:]], 1)
    assert _rel_err(out, ref) < 1e-2


@pytest.mark.parametrize("variant", VARIANTS)
@pytest.mark.parametrize("I", [2624, 2600, 384])
def test_gemm_geglu_epilogue(cuda_lib, I, variant):
    from sys1rust_b200.backend import EPI_GEGLU, gemm, interleave_wi
    if variant == 5:
        pytest.skip("GeGLU tiles are 256 wide")
    M, K = 260, 1024
    a = _rand((M, K), 11)
    wi = _rand((2 * I, K), 12)
    wil = torch.from_numpy(interleave_wi(wi.cpu().view(torch.int16).numpy(), I)).view(torch.bfloat16).cuda()
    out = torch.empty(M, I, dtype=torch.bfloat16, device="cuda")
    gemm(EPI_GEGLU, a.data_ptr(), wil.data_ptr(), out.data_ptr(), M, wil.shape[0], K, out_cols=I, variant=variant)
    torch.cuda.synchronize()
    y = a.float() @ wi.float().t()
    ref = torch.nn.functional.gelu(y[:, :I]) * y[:, I:]
    assert _rel_err(out, ref) < 1e-2


def _attn_ref(q, k, v, cu, window, scale, heads):
    out = torch.zeros_like(q, dtype=torch.float32)
    for r in range(len(cu) - 1):
        s, e = int(cu[r]), int(cu[r + 1])
        L = e - s
        qh = q[s:e].float().view(L, heads, 64).transpose(0, 1)
        kh = k[s:e].float().view(L, heads, 64).transpose(0, 1)
        vh = v[s:e].float().view(L, heads, 64).transpose(0, 1)
        sc = qh @ kh.transpose(1, 2) * scale
        if window >= 0:
            p = torch.arange(L, device=q.device)
            sc = sc.masked_fill((p[:, None] - p[None, :]).abs() > window, float("-inf"))
        out[s:e] = (torch.softmax(sc, -1) @ vh).transpose(0, 1).reshape(L, heads * 64)
    return out


@pytest.mark.parametrize("impl", [1, 0])
@pytest.mark.parametrize("window", [-1, 64, 3])
def test_attention_varlen_matches_torch(cuda_lib, window, impl):
    from sys1rust_b200.backend import attention
    heads, d = 16, 1024
    lens = [1, 2, 63, 64, 65, 129, 300, 1024]
    cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    T = int(cu[-1])
    qkv = _rand((T, 3 * d), 13)
    o = torch.empty(T, d, dtype=torch.bfloat16, device="cuda")
    attention(qkv.data_ptr(), qkv[:, d:].data_ptr(), qkv[:, 2 * d:].data_ptr(), o.data_ptr(), 3 * d, 3 * d, 3 * d, d,
              heads, cu, window, 0.125, impl=impl)
    ref = _attn_ref(qkv[:, :d], qkv[:, d:2 * d], qkv[:, 2 * d:], cu, window, 0.125, heads)
    assert _rel_err(o, ref) < 1e-2


@pytest.mark.parametrize("window", [-1, 64])
def test_attention_many_units_per_cta(cuda_lib, window):
    """The persistent tcgen05 kernel with several units per CTA: 60 sequences of 17..700 tokens
    (~180 query tiles x 16 heads, about ten units for each of the 296 CTAs), so the Q and O
    buffers alternate across units of different lengths and the deferred epilogue of one unit
    runs inside the next; against torch fp32."""
    from sys1rust_b200.backend import attention
    heads, d = 16, 1024
    rng = np.random.default_rng(5)
    lens = [int(x) for x in rng.integers(17, 700, size=60)]
    cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    T = int(cu[-1])
    qkv = _rand((T, 3 * d), 51)
    o = torch.empty(T, d, dtype=torch.bfloat16, device="cuda")
    attention(qkv.data_ptr(), qkv[:, d:].data_ptr(), qkv[:, 2 * d:].data_ptr(), o.data_ptr(), 3 * d, 3 * d, 3 * d, d,
              heads, cu, window, 0.125, impl=0)
    ref = _attn_ref(qkv[:, :d], qkv[:, d:2 * d], qkv[:, 2 * d:], cu, window, 0.125, heads)
    assert _rel_err(o, ref) < 1e-2


@pytest.mark.parametrize("impl", [1, 0])
@pytest.mark.parametrize("window", [-1, 64])
def test_attention_growing_scores(cuda_lib, window, impl):
    """Scores with a spread of tens (q, k scaled by 4) whose maximum grows along the row (keys
    scaled by 1 + 3 j / L): the running maximum rises by more than 2^8 between key tiles, so the
    tcgen05 kernel's rescale of the TMEM accumulator runs (and the mma.sync kernel's correction)."""
    from sys1rust_b200.backend import attention
    heads, d = 16, 1024
    lens = [70, 200, 513, 1024]
    cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    T = int(cu[-1])
    qkv = _rand((T, 3 * d), 29).float()
    ramp = torch.cat([1 + 3 * torch.arange(L, dtype=torch.float32, device="cuda") / L for L in lens])
    qkv[:, :d] *= 4
    qkv[:, d:2 * d] *= 4 * ramp[:, None]
    qkv = qkv.to(torch.bfloat16)
    o = torch.empty(T, d, dtype=torch.bfloat16, device="cuda")
    attention(qkv.data_ptr(), qkv[:, d:].data_ptr(), qkv[:, 2 * d:].data_ptr(), o.data_ptr(), 3 * d, 3 * d, 3 * d, d,
              heads, cu, window, 0.125, impl=impl)
    ref = _attn_ref(qkv[:, :d], qkv[:, d:2 * d], qkv[:, 2 * d:], cu, window, 0.125, heads)
    assert torch.isfinite(o.float()).all()
    assert _rel_err(o, ref) < 1e-2
