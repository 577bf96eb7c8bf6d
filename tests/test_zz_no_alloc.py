"""The allocation-free split-K GEMM (``s1c_gemm_splitk_noalloc``) against a plain PyTorch fp32
product with the same epilogue and against the split-K path of ``s1c_gemm`` (variant 3), through
the C ABI.

Some callers cannot allocate device memory: a serving loop that must not stall in cudaMalloc or
cudaFree (both can synchronise the whole device), or a host whose framework owns all device memory
through its own pool. For them the split-K partial sums live in a fixed 4 MiB array compiled into
the library. This file is collected last so that, if it fails, a run that stops at the first
failure has already run every other test; it also passes on its own in a fresh process.
Tolerances are those of the kernel tests: ``max|out - ref| <= 1e-2 * max|ref|`` for bf16 outputs,
1e-4 for fp32 outputs (the two paths may split K differently, so sums are rounded differently).
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")
F = torch.nn.functional

pytestmark = pytest.mark.gpu


def _rel_err(out, ref):
    return (out.float() - ref.float()).abs().max().item() / max(ref.float().abs().max().item(), 1e-30)


def _rand(shape, seed):
    g = torch.Generator(device="cpu").manual_seed(seed)
    return torch.randn(*shape, generator=g).to(torch.bfloat16).cuda()


@pytest.fixture(scope="module")
def lib_built():
    from sys1rust_b200 import build
    build.build()
    from sys1rust_b200.backend import lib
    return lib()


def _rope_ref(x, pos, theta):
    """Rotate-half RoPE per 64-wide head of x [M, C] at positions pos [M]: pairs (i, i + 32) turned
    by pos * theta^(-i/32), the angle formed in fp32 (split_rope.metal:46-76)."""
    M, C = x.shape
    lbase = torch.log2(torch.tensor(theta, dtype=torch.float32))
    inv = torch.exp2(-(torch.arange(32, dtype=torch.float32) / 32) * lbase)
    ang = pos.float().cpu()[:, None] * inv[None, :]
    c, s = torch.cos(ang).cuda()[:, None], torch.sin(ang).cuda()[:, None]
    xh = x.view(M, C // 64, 64)
    x1, x2 = xh[..., :32], xh[..., 32:]
    return torch.cat([x1 * c - x2 * s, x1 * s + x2 * c], -1).view(M, C)


def _case(case, M, K):
    """(epi, B operand, kwargs, fresh output, fp32 reference) of one epilogue case."""
    from sys1rust_b200.backend import EPI_GEGLU, EPI_RESID, EPI_ROPE, EPI_STORE, interleave_wi
    a = _rand((M, K), 41)
    kw = {}
    if case == "geglu":
        I = 384
        wi = _rand((2 * I, K), 42)
        b = torch.from_numpy(interleave_wi(wi.cpu().view(torch.int16).numpy(), I)).view(torch.bfloat16).cuda()
        epi, kw = EPI_GEGLU, {"out_cols": I}
        mk = lambda: torch.empty(M, I, dtype=torch.bfloat16, device="cuda")
        y = a.float() @ wi.float().t()
        ref = F.gelu(y[:, :I]) * y[:, I:]
    elif case.startswith("rope"):
        theta = 10000.0 if case == "rope" else 160000.0
        N, epi = 768, EPI_ROPE
        b = _rand((N, K), 43)
        pos = torch.from_numpy((np.arange(M) % 150).astype(np.int32)).cuda()
        kw = {"pos_ptr": pos.data_ptr(), "rope_theta": theta, "rope_cols": 512, "_keep": pos}
        mk = lambda: torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
        acc = a.float() @ b.float().t()
        ref = torch.cat([_rope_ref(acc[:, :512], pos, theta), acc[:, 512:]], 1)
    elif case == "resid":
        N, epi = 1024, EPI_RESID
        b = _rand((N, K), 44)
        h0 = torch.randn(M, N, generator=torch.Generator().manual_seed(45)).float().cuda()
        mk = lambda: h0.clone()
        ref = h0 + a.float() @ b.float().t()
    else:
        N, epi = 512, EPI_STORE
        b = _rand((N, K), 46)
        ref = a.float() @ b.float().t()
        if case == "store_f32_gelu":
            bias = torch.randn(N, generator=torch.Generator().manual_seed(47)).float().cuda()
            kw = {"bias_ptr": bias.data_ptr(), "act": 2, "out_f32": 1, "_keep": bias}
            mk = lambda: torch.empty(M, N, dtype=torch.float32, device="cuda")
            ref = F.gelu(ref + bias)
        else:
            mk = lambda: torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
    return a, epi, b, kw, mk, ref


def _call(fn, epi, a, b, out, M, K, kw, **extra):
    args = {k: v for k, v in kw.items() if not k.startswith("_")}
    fn(epi, a.data_ptr(), b.data_ptr(), out.data_ptr(), M, b.shape[0], K, **args, **extra)


@pytest.mark.parametrize("case", ["store", "store_f32_gelu", "resid", "geglu", "rope", "rope_global"])
def test_noalloc_matches_fp32_and_split_k_entry_point(lib_built, case):
    from sys1rust_b200.backend import gemm, gemm_splitk_noalloc
    M, K = 200, 1024
    a, epi, b, kw, mk, ref32 = _case(case, M, K)
    ref = mk()
    _call(gemm, epi, a, b, ref, M, K, kw, variant=3)
    torch.cuda.synchronize()
    tol = 1e-4 if ref.dtype == torch.float32 else 1e-2
    for _ in range(2):  # two calls in a row share (and overwrite) the static scratch
        out = mk()
        _call(gemm_splitk_noalloc, epi, a, b, out, M, K, kw)
        torch.cuda.synchronize()
        assert torch.isfinite(out.float()).all()
        assert _rel_err(out, ref32) < tol  # the plain fp32 product with the same epilogue
        assert _rel_err(out, ref) < tol    # the split-K entry point that allocates its workspace


def test_noalloc_calls_allocate_no_device_memory(lib_built):
    """Free device memory is the same before and after calls of every epilogue (RoPE with a theta
    not used before included), once each kind of call has run once (the CUDA runtime loads a
    kernel's module at its first launch)."""
    from sys1rust_b200.backend import gemm_splitk_noalloc
    M, K = 200, 1024
    cases = [_case(c, M, K) for c in ("store", "store_f32_gelu", "resid", "geglu", "rope")]
    outs = [mk() for (_, _, _, _, mk, _) in cases]
    for (a, epi, b, kw, _, _), out in zip(cases, outs):
        _call(gemm_splitk_noalloc, epi, a, b, out, M, K, kw)
    torch.cuda.synchronize()
    free0 = torch.cuda.mem_get_info()[0]
    for rep in range(3):
        for (a, epi, b, kw, _, _), out in zip(cases, outs):
            if "rope_theta" in kw:
                kw = {**kw, "rope_theta": 5000.0 + 1000.0 * rep}
            _call(gemm_splitk_noalloc, epi, a, b, out, M, K, kw)
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info()[0] == free0


def test_noalloc_rejects_sizes_past_the_scratch(lib_built):
    """Two split slices of 1024 x 1024 fp32 need 8 MiB: refused before anything is launched."""
    from sys1rust_b200.backend import BackendError, EPI_STORE, gemm_splitk_noalloc
    with pytest.raises(BackendError, match="static scratch"):
        gemm_splitk_noalloc(EPI_STORE, 16, 16, 16, 1024, 1024, 1024)
