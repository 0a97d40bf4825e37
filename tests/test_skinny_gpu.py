"""Few-row (swap-AB) tcgen05 GEMM against fp32 PyTorch matmuls of the same bf16
inputs: dense shapes of a decode step (1..128 token rows, weights up to
9216 x 8192, ragged N and K), every epilogue, the grouped form with packed
per-expert row ranges (empty experts, one expert holding every row), and the
inference MoE path against the training (autograd) path."""
import pytest
import torch

pytestmark = pytest.mark.gpu

EPI_BF16, EPI_F32, EPI_ACC, EPI_ADD, EPI_SWIGLU, EPI_SWIGLU_BWD = range(6)


def _rel(a, b):
    return ((a.float() - b.float()).abs().max() / (b.float().abs().max() + 1e-6)).item()


def _mk(*shape, scale=1.0):
    return (torch.randn(*shape, device="cuda") * scale).to(torch.bfloat16)


@pytest.mark.parametrize("M,N,K", [(1, 576, 2048), (7, 2048, 8192), (16, 9216, 2048), (64, 2816, 2048),
                                   (100, 300, 200), (128, 1000, 136), (33, 32000, 1024)])
def test_skinny_dense_store(cuda_ext, M, N, K):
    torch.manual_seed(0)
    A, B = _mk(M, K), _mk(N, K, scale=0.05)
    C = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    cuda_ext.gemm(A, B, C, False, False, EPI_BF16, 1.0, None, None, 256)
    assert _rel(C, A.float() @ B.float().T) < 1e-2
    C32 = torch.empty(M, N, device="cuda", dtype=torch.float32)
    cuda_ext.gemm(A, B, C32, False, False, EPI_F32, 0.5, None, None, 256)
    assert _rel(C32, 0.5 * (A.float() @ B.float().T)) < 1e-3


def test_skinny_dense_residual_and_swiglu(cuda_ext):
    torch.manual_seed(1)
    M, N, K = 48, 2048, 1408
    A, B, R = _mk(M, K), _mk(N, K, scale=0.05), _mk(M, N)
    C = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    cuda_ext.gemm(A, B, C, False, False, EPI_ADD, 1.0, R, None, 256)
    assert _rel(C, A.float() @ B.float().T + R.float()) < 1e-2
    W13 = _mk(2 * 1408, 2048, scale=0.05)
    X = _mk(M, 2048)
    act = torch.empty(M, 1408, device="cuda", dtype=torch.bfloat16)
    cuda_ext.gemm(X, W13, act, False, False, EPI_SWIGLU, 1.0, None, None, 256)
    h = (X.float() @ W13.float().T).view(M, -1, 2, 32)
    ref = (torch.nn.functional.silu(h[:, :, 0]) * h[:, :, 1]).reshape(M, 1408)
    assert _rel(act, ref) < 1e-2


def test_skinny_matches_tile_gemm(cuda_ext):
    """The same product through the few-row kernel and through the tile GEMM."""
    torch.manual_seed(2)
    A, B = _mk(64, 2048), _mk(4096, 2048, scale=0.05)
    c1 = torch.empty(64, 4096, device="cuda", dtype=torch.float32)
    c2 = torch.empty_like(c1)
    cuda_ext.gemm(A, B, c1, False, False, EPI_F32, 1.0, None, None, 256)
    cuda_ext.set_skinny_rows(0)
    try:
        cuda_ext.gemm(A, B, c2, False, False, EPI_F32, 1.0, None, None, 256)
    finally:
        cuda_ext.set_skinny_rows(128)
    assert _rel(c1, c2) < 1e-4


@pytest.mark.parametrize("counts", [[3, 0, 17, 1, 0, 64, 9, 2], [0, 0, 0, 100, 0, 0, 0, 0], [1] * 8])
def test_skinny_grouped(cuda_ext, counts):
    torch.manual_seed(3)
    E, D, F = len(counts), 1024, 704
    n = sum(counts)
    off = torch.tensor([0] + list(torch.tensor(counts).cumsum(0)), dtype=torch.int32, device="cuda")
    X = _mk(n, D)
    W13 = _mk(E, 2 * F, D, scale=0.05)
    W2 = _mk(E, D, F, scale=0.05)
    act = torch.empty(n, F, device="cuda", dtype=torch.bfloat16)
    cuda_ext.gemm_skinny_grouped(X, W13, off, act, EPI_SWIGLU, 1.0, n)
    y = torch.empty(n, D, device="cuda", dtype=torch.bfloat16)
    cuda_ext.gemm_skinny_grouped(act, W2, off, y, EPI_BF16, 1.0, n)
    ref_act, ref_y = [], []
    for e in range(E):
        a, b = int(off[e]), int(off[e + 1])
        if b == a:
            continue
        h = (X[a:b].float() @ W13[e].float().T).view(b - a, -1, 2, 32)
        g = (torch.nn.functional.silu(h[:, :, 0]) * h[:, :, 1]).reshape(b - a, F)
        ref_act.append(g)
        ref_y.append(act[a:b].float() @ W2[e].float().T)
    assert _rel(act, torch.cat(ref_act)) < 1e-2
    assert _rel(y, torch.cat(ref_y)) < 1e-2


@pytest.mark.parametrize("T", [16, 64, 200])
def test_moe_inference_path_matches_training_path(cuda_ext, T):
    from omnicoder.ops.moe import moe_ffn
    torch.manual_seed(4)
    E, D, F, k = 32, 512, 256, 4
    x = _mk(T, D)
    rw = _mk(E, D, scale=0.1)
    w13 = _mk(E, 2 * F, D, scale=0.05)
    w2 = _mk(E, D, F, scale=0.05)
    with torch.no_grad():
        y_inf, _ = moe_ffn(x, rw, w13, w2, k)
    xg = x.clone().requires_grad_(True)
    y_tr, _ = moe_ffn(xg, rw, w13, w2, k)
    assert _rel(y_inf, y_tr.detach()) < 2e-2


@pytest.mark.gpu
def test_few_row_library_route(cuda_ext):
    """Plain few-row projections (decode steps) on the library GEMM, with and without the residual,
    against the fp32 product; more rows stay on the tcgen05 kernels."""
    from omnicoder.ops import gemm as G
    assert G.FEW_ROW_LIBRARY_MAX >= 64
    torch.manual_seed(0)
    for M in (1, 37, 64):
        x = torch.randn(M, 2048, device="cuda").to(torch.bfloat16)
        w = (0.02 * torch.randn(576, 2048, device="cuda")).to(torch.bfloat16)
        r = torch.randn(M, 576, device="cuda").to(torch.bfloat16)
        ref = x.float() @ w.float().t()
        assert (G.mm_nt(x, w).float() - ref).abs().max() / ref.abs().max() < 1e-2
        assert (G.mm_nt(x, w, residual=r).float() - (ref + r.float())).abs().max() / ref.abs().max() < 2e-2
