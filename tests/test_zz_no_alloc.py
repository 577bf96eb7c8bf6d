"""The allocation-free split-K GEMM (``s1c_gemm_splitk_noalloc``) against the split-K path of
``s1c_gemm`` (variant 3), through the C ABI.

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


@pytest.mark.parametrize("case", ["store", "store_f32_gelu", "resid", "geglu", "rope"])
def test_noalloc_matches_split_k_entry_point(lib_built, case):
    from sys1rust_b200.backend import (EPI_GEGLU, EPI_RESID, EPI_ROPE, EPI_STORE, gemm, gemm_splitk_noalloc,
                                       interleave_wi)
    M, K = 200, 1024
    a = _rand((M, K), 41)
    kw = {}
    if case == "geglu":
        I = 384
        wi = _rand((2 * I, K), 42)
        b = torch.from_numpy(interleave_wi(wi.cpu().view(torch.int16).numpy(), I)).view(torch.bfloat16).cuda()
        N, epi, kw = b.shape[0], EPI_GEGLU, {"out_cols": I}
        mk = lambda: torch.empty(M, I, dtype=torch.bfloat16, device="cuda")
    elif case == "rope":
        N, epi = 768, EPI_ROPE
        b = _rand((N, K), 43)
        pos = torch.from_numpy((np.arange(M) % 150).astype(np.int32)).cuda()
        kw = {"pos_ptr": pos.data_ptr(), "rope_theta": 10000.0, "rope_cols": 512}
        mk = lambda: torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
    elif case == "resid":
        N, epi = 1024, EPI_RESID
        b = _rand((N, K), 44)
        h0 = torch.randn(M, N, generator=torch.Generator().manual_seed(45)).float().cuda()
        mk = lambda: h0.clone()
    else:
        N, epi = 512, EPI_STORE
        b = _rand((N, K), 46)
        if case == "store_f32_gelu":
            bias = torch.randn(N, generator=torch.Generator().manual_seed(47)).float().cuda()
            kw = {"bias_ptr": bias.data_ptr(), "act": 2, "out_f32": 1}
            mk = lambda: torch.empty(M, N, dtype=torch.float32, device="cuda")
        else:
            mk = lambda: torch.empty(M, N, dtype=torch.bfloat16, device="cuda")
    ref = mk()
    gemm(epi, a.data_ptr(), b.data_ptr(), ref.data_ptr(), M, N, K, variant=3, **kw)
    torch.cuda.synchronize()
    tol = 1e-4 if ref.dtype == torch.float32 else 1e-2
    for _ in range(2):  # two calls in a row share (and overwrite) the static scratch
        out = mk()
        gemm_splitk_noalloc(epi, a.data_ptr(), b.data_ptr(), out.data_ptr(), M, N, K, **kw)
        torch.cuda.synchronize()
        assert torch.isfinite(out.float()).all()
        assert _rel_err(out, ref) < tol


def test_noalloc_rejects_sizes_past_the_scratch(lib_built):
    """Two split slices of 1024 x 1024 fp32 need 8 MiB: refused before anything is launched."""
    from sys1rust_b200.backend import BackendError, EPI_STORE, gemm_splitk_noalloc
    with pytest.raises(BackendError, match="static scratch"):
        gemm_splitk_noalloc(EPI_STORE, 16, 16, 16, 1024, 1024, 1024)
