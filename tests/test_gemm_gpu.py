"""tcgen05 GEMM numerics against a plain fp32 PyTorch matmul of the same bf16 inputs."""
import pytest
import torch

pytestmark = pytest.mark.gpu

EPI_BF16, EPI_F32, EPI_ACC, EPI_ADD, EPI_SWIGLU, EPI_SWIGLU_BWD = range(6)


def _rel(a, b):
    return ((a.float() - b.float()).abs().max() / (b.float().abs().max() + 1e-6)).item()


def _rowrel(a, b):
    """Per-row relative error ||a - b|| / ||b||: (mean, max).  A wrong small-magnitude region, which
    the max-abs / max-ref ratio can hide, shows up here at ~1."""
    a, b = a.float().reshape(-1, a.shape[-1]), b.float().reshape(-1, b.shape[-1])
    r = (a - b).norm(dim=-1) / (b.norm(dim=-1) + 1e-6)
    return r.mean().item(), r.max().item()


def _mk(*shape, scale=1.0):
    return (torch.randn(*shape, device="cuda") * scale).to(torch.bfloat16)


@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (256, 512, 256), (300, 520, 200), (1024, 768, 1408), (64, 32, 32)])
@pytest.mark.parametrize("block_n", [128, 256])
def test_dense_kk(cuda_ext, M, N, K, block_n):
    torch.manual_seed(0)
    A, B = _mk(M, K), _mk(N, K)
    C = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    cuda_ext.gemm(A, B, C, False, False, EPI_BF16, 1.0, None, None, block_n)
    ref = A.float() @ B.float().T
    assert _rel(C, ref) < 1e-2


@pytest.mark.parametrize("M,N,K", [(256, 512, 384), (200, 136, 128), (512, 2048, 1408)])
def test_dense_k_mn(cuda_ext, M, N, K):
    # dX = dY @ W  with W stored [K_red, N]
    torch.manual_seed(1)
    A, B = _mk(M, K), _mk(K, N)
    C = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    cuda_ext.gemm(A, B, C, False, True, EPI_BF16, 1.0, None, None, 256)
    ref = A.float() @ B.float()
    assert _rel(C, ref) < 1e-2


@pytest.mark.parametrize("M,N,K", [(256, 512, 384), (192, 320, 1000), (2048, 1408, 512)])
def test_dense_mn_mn(cuda_ext, M, N, K):
    # dW = dY^T X with dY [K_red, M], X [K_red, N]
    torch.manual_seed(2)
    A, B = _mk(K, M), _mk(K, N)
    C = torch.empty(M, N, device="cuda", dtype=torch.float32)
    cuda_ext.gemm(A, B, C, True, True, EPI_F32, 0.5, None, None, 256)
    ref = 0.5 * (A.float().T @ B.float())
    assert _rel(C, ref) < 2e-3
    C2 = C.clone()
    cuda_ext.gemm(A, B, C2, True, True, EPI_ACC, 1.0, None, None, 128)
    assert _rel(C2, C + ref / 0.5) < 2e-3
    Cb = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    cuda_ext.gemm(A, B, Cb, True, True, EPI_BF16, 1.0, None, None, 256)
    assert _rel(Cb, ref / 0.5) < 1e-2


def test_dense_add_residual(cuda_ext):
    torch.manual_seed(3)
    A, B, R = _mk(384, 512), _mk(256, 512), _mk(384, 256)
    C = torch.empty(384, 256, device="cuda", dtype=torch.bfloat16)
    cuda_ext.gemm(A, B, C, False, False, EPI_ADD, 1.0, R, None, 256)
    ref = A.float() @ B.float().T + R.float()
    assert _rel(C, ref) < 1e-2
    # in place: C = acc + C
    C2 = R.clone()
    cuda_ext.gemm(A, B, C2, False, False, EPI_ADD, 1.0, C2, None, 256)
    assert _rel(C2, ref) < 1e-2


def _interleave(w1, w3, blk=32):
    F, D = w1.shape
    return torch.stack([w1.view(F // blk, blk, D), w3.view(F // blk, blk, D)], 1).reshape(2 * F, D)


def test_dense_swiglu_fwd_bwd(cuda_ext):
    torch.manual_seed(4)
    T, D, F = 256, 512, 384
    x = _mk(T, D)
    w1, w3 = _mk(F, D, scale=0.05), _mk(F, D, scale=0.05)
    w13 = _interleave(w1, w3)
    act = torch.empty(T, F, device="cuda", dtype=torch.bfloat16)
    H = torch.empty(T, 2 * F, device="cuda", dtype=torch.bfloat16)
    cuda_ext.gemm(x, w13, act, False, False, EPI_SWIGLU, 1.0, None, H, 256)
    g = x.float() @ w1.float().T
    u = x.float() @ w3.float().T
    ref = torch.nn.functional.silu(g) * u
    assert _rel(act, ref) < 2e-2
    assert _rel(H, x.float() @ w13.float().T) < 1e-2
    # backward: dAct = dY @ W2 ; dH = swiglu'(H) * dAct
    w2 = _mk(D, F, scale=0.05)
    dy = _mk(T, D)
    dH = torch.empty(T, 2 * F, device="cuda", dtype=torch.bfloat16)
    cuda_ext.gemm(dy, w2, dH, False, True, EPI_SWIGLU_BWD, 1.0, H, None, 256)
    da = dy.float() @ w2.float()
    Hf = H.float().view(T, F // 32, 2, 32)
    gg, uu = Hf[:, :, 0].reshape(T, F), Hf[:, :, 1].reshape(T, F)
    sg = torch.sigmoid(gg)
    dg = da * uu * sg * (1 + gg * (1 - sg))
    du = da * gg * sg
    ref_dh = torch.stack([dg.view(T, F // 32, 32), du.view(T, F // 32, 32)], 2).reshape(T, 2 * F)
    assert _rel(dH, ref_dh) < 2e-2
    mean, worst = _rowrel(dH, ref_dh)
    assert mean < 2e-2 and worst < 8e-2, (mean, worst)


def _offsets(counts):
    pad = [(c + 127) // 128 * 128 for c in counts]
    off = [0]
    for p in pad:
        off.append(off[-1] + p)
    return off


@pytest.mark.parametrize("b_mn", [False, True])
def test_grouped_m(cuda_ext, b_mn):
    torch.manual_seed(5)
    G, N, K = 5, 384, 256
    counts = [130, 0, 7, 256, 300]
    off = _offsets(counts)
    rows = off[-1] + 128
    A = torch.zeros(rows, K, device="cuda", dtype=torch.bfloat16)
    for g in range(G):
        A[off[g]:off[g] + counts[g]] = _mk(counts[g], K)
    B = _mk(G, K, N) if b_mn else _mk(G, N, K)
    offs = torch.tensor(off, device="cuda", dtype=torch.int32)
    C = torch.full((rows, N), 7.0, device="cuda", dtype=torch.bfloat16)
    cuda_ext.gemm_grouped_m(A, B, offs, C, b_mn, EPI_BF16, 1.0, None, None, 256, rows)
    for g in range(G):
        Bg = B[g].float() if b_mn else B[g].float().T
        ref = A[off[g]:off[g + 1]].float() @ Bg
        if off[g + 1] > off[g]:
            assert _rel(C[off[g]:off[g + 1]], ref) < 1e-2, g


def test_grouped_k(cuda_ext):
    torch.manual_seed(6)
    G, M, N = 4, 256, 384
    counts = [128, 0, 250, 513]
    off = _offsets(counts)
    rows = off[-1]
    A = torch.zeros(rows, M, device="cuda", dtype=torch.bfloat16)
    B = torch.zeros(rows, N, device="cuda", dtype=torch.bfloat16)
    for g in range(G):
        A[off[g]:off[g] + counts[g]] = _mk(counts[g], M)
        B[off[g]:off[g] + counts[g]] = _mk(counts[g], N)
    offs = torch.tensor(off, device="cuda", dtype=torch.int32)
    C = torch.full((G, M, N), 3.0, device="cuda", dtype=torch.bfloat16)
    cuda_ext.gemm_grouped_k(A, B, offs, C, EPI_BF16, 1.0, 256)
    for g in range(G):
        ref = A[off[g]:off[g + 1]].float().T @ B[off[g]:off[g + 1]].float()
        if counts[g] == 0:
            assert C[g].abs().max().item() == 0.0
        else:
            assert _rel(C[g], ref) < 1e-2, g


@pytest.mark.parametrize("layout", ["kk", "k_mn", "mn_mn"])
@pytest.mark.parametrize("M,N,K", [(4096, 4096, 256), (384, 768, 640), (1000, 264, 136)])
def test_cta_pair_tiles_match_single_cta(cuda_ext, layout, M, N, K):
    """256-row CTA-pair tiles (cta_group::2) give the one-CTA kernel's result, including
    ragged M / N / K edges and more tiles than co-resident pairs."""
    torch.manual_seed(7)
    a_mn, b_mn = {"kk": (False, False), "k_mn": (False, True), "mn_mn": (True, True)}[layout]
    A = _mk(K, M) if a_mn else _mk(M, K)
    B = _mk(K, N) if b_mn else _mk(N, K)
    f32 = layout != "k_mn"                  # the (K, MN) layout has bf16 epilogues only
    out = []
    try:
        for pair in (False, True):
            cuda_ext.set_gemm_pair(pair)
            C = torch.empty(M, N, device="cuda", dtype=torch.float32 if f32 else torch.bfloat16)
            cuda_ext.gemm(A, B, C, a_mn, b_mn, EPI_F32 if f32 else EPI_BF16, 1.0, None, None, 256)
            out.append(C)
    finally:
        cuda_ext.set_gemm_pair(True)
    ref = (A.float().T if a_mn else A.float()) @ (B.float() if b_mn else B.float().T)
    assert _rel(out[1], ref) < (2e-3 if f32 else 1e-2)
    assert _rel(out[1], out[0]) < (1e-5 if f32 else 1e-2)


def test_cta_pair_grouped_k(cuda_ext):
    torch.manual_seed(8)
    G, M, N = 3, 640, 512
    counts = [384, 0, 1000]
    off = _offsets(counts)
    rows = off[-1]
    A = torch.zeros(rows, M, device="cuda", dtype=torch.bfloat16)
    B = torch.zeros(rows, N, device="cuda", dtype=torch.bfloat16)
    for g in range(G):
        A[off[g]:off[g] + counts[g]] = _mk(counts[g], M)
        B[off[g]:off[g] + counts[g]] = _mk(counts[g], N)
    offs = torch.tensor(off, device="cuda", dtype=torch.int32)
    assert cuda_ext.gemm_pair_enabled()
    C = torch.full((G, M, N), 3.0, device="cuda", dtype=torch.float32)
    cuda_ext.gemm_grouped_k(A, B, offs, C, EPI_F32, 1.0, 256)
    for g in range(G):
        ref = A[off[g]:off[g + 1]].float().T @ B[off[g]:off[g + 1]].float()
        assert _rel(C[g], ref) < 2e-3 if counts[g] else C[g].abs().max().item() == 0.0


@pytest.mark.parametrize("ldc_pad", [0, 8])
def test_bf16_epilogue_strided_output(cuda_ext, ldc_pad):
    """bf16 outputs leave through shared memory + TMA stores into a strided view; columns
    past N stay untouched."""
    torch.manual_seed(9)
    M, N, K = 640, 320, 512
    A, B = _mk(M, K), _mk(N, K)
    full = torch.full((M, N + ldc_pad), 5.0, device="cuda", dtype=torch.bfloat16)
    C = full[:, :N]
    cuda_ext.gemm(A, B, C, False, False, EPI_BF16, 1.0, None, None, 256)
    assert _rel(C, A.float() @ B.float().T) < 1e-2
    if ldc_pad:
        assert (full[:, N:] == 5.0).all()


def test_unaligned_output_rows_are_rejected(cuda_ext):
    """An output whose rows do not start on 16-byte boundaries is refused on the host
    (the epilogue writes 16-byte vectors); nothing is launched."""
    A, B = _mk(256, 64), _mk(320, 64)
    C = torch.zeros(256, 325, device="cuda", dtype=torch.bfloat16)[:, :320]
    with pytest.raises(RuntimeError, match="16-byte"):
        cuda_ext.gemm(A, B, C, False, False, EPI_BF16, 1.0, None, None, 256)
    torch.cuda.synchronize()


def test_swiglu_epilogue_partial_tile(cuda_ext):
    """SwiGLU outputs (activation and saved pre-activation) on a tile that overhangs N and M."""
    torch.manual_seed(10)
    T, D, F = 200, 256, 96                  # 2F = 192 accumulator columns: one partial 256-wide tile
    x = _mk(T, D)
    w1, w3 = _mk(F, D, scale=0.05), _mk(F, D, scale=0.05)
    w13 = _interleave(w1, w3)
    act = torch.empty(T, F, device="cuda", dtype=torch.bfloat16)
    H = torch.empty(T, 2 * F, device="cuda", dtype=torch.bfloat16)
    cuda_ext.gemm(x, w13, act, False, False, EPI_SWIGLU, 1.0, None, H, 256)
    ref = torch.nn.functional.silu(x.float() @ w1.float().T) * (x.float() @ w3.float().T)
    assert _rel(act, ref) < 2e-2
    assert _rel(H, x.float() @ w13.float().T) < 1e-2


@pytest.mark.parametrize("inplace", [False, True])
def test_residual_epilogue_ragged(cuda_ext, inplace):
    """Residual epilogue (R boxes loaded by TMA one chunk ahead) on tiles overhanging M and N."""
    torch.manual_seed(11)
    M, N, K = 300, 200, 256
    A, B, R = _mk(M, K), _mk(N, K), _mk(M, N)
    ref = A.float() @ B.float().T + R.float()
    C = R.clone() if inplace else torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
    cuda_ext.gemm(A, B, C, False, False, EPI_ADD, 1.0, C if inplace else R, None, 256)
    assert _rel(C, ref) < 1e-2


def test_grouped_m_swiglu_bwd(cuda_ext):
    """SwiGLU-backward epilogue of the grouped expert GEMM (H boxes loaded by TMA)."""
    torch.manual_seed(12)
    G, D, F = 3, 256, 192
    counts = [130, 0, 256]
    off = _offsets(counts)
    rows = off[-1]
    dy = torch.zeros(rows, D, device="cuda", dtype=torch.bfloat16)
    H = torch.zeros(rows, 2 * F, device="cuda", dtype=torch.bfloat16)
    for g in range(G):
        dy[off[g]:off[g] + counts[g]] = _mk(counts[g], D)
        H[off[g]:off[g] + counts[g]] = _mk(counts[g], 2 * F)
    w2 = _mk(G, D, F, scale=0.05)                          # [G, K = D, N = F]
    offs = torch.tensor(off, device="cuda", dtype=torch.int32)
    dH = torch.zeros(rows, 2 * F, device="cuda", dtype=torch.bfloat16)
    cuda_ext.gemm_grouped_m(dy, w2, offs, dH, True, EPI_SWIGLU_BWD, 1.0, H, None, 256, rows)
    for g in range(G):
        if counts[g] == 0:
            continue
        sl = slice(off[g], off[g] + counts[g])
        da = dy[sl].float() @ w2[g].float()
        Hf = H[sl].float().view(-1, F // 32, 2, 32)
        gg, uu = Hf[:, :, 0].reshape(-1, F), Hf[:, :, 1].reshape(-1, F)
        sg = torch.sigmoid(gg)
        dg = da * uu * sg * (1 + gg * (1 - sg))
        du = da * gg * sg
        ref = torch.stack([dg.view(-1, F // 32, 32), du.view(-1, F // 32, 32)], 2).reshape(-1, 2 * F)
        assert _rel(dH[sl], ref) < 2e-2, g
        mean, worst = _rowrel(dH[sl], ref)
        assert mean < 2e-2 and worst < 8e-2, (g, mean, worst)
