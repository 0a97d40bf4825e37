"""Block-scaled fp8 (e4m3) linear algebra: 1 x 128 activation scales and
128 x 128 weight scales, the tile scheme of block-scaled fp8 training recipes.

  quantize_act(x [M, K])         -> (xq e4m3 [M, K], sx fp32 [K/128, M padded to 128])
  quantize_weight(w [(G,) N, K]) -> (wq e4m3, sw fp32 [G, ceil(N/128), K/128])
  fp8_mm(x, wq, sw)              -> x @ dequant(w)^T in bf16 (x quantised on the fly)
  fp8_grouped_mm(x_perm, wq, sw, offsets, rows) -> per-expert products (row groups of
                                    x_perm given by offsets, multiples of 128)

Scales are max|block| / 448 (e4m3's largest finite value) rounded up to a power of two
(`pow2=True`, the default; an all-zero block gets scale 1).  A power-of-two scale is an
8-bit exponent (UE8M0), so the CUDA GEMM hands the scales to the tensor core
(tcgen05 kind::mxf8f6f4 block-scaled MMA, each 128-block scale repeated over its four
32-wide slices) and accumulates all K blocks in tensor memory.  With `pow2=False` the
scales are exact fp32 ratios and the GEMM must be called with `scaled_mma=False`: then
each 128-wide K block's partial product is scaled and accumulated in fp32 by the
epilogue warps (gemm_fp8.cu).  CPU: dequantise and matmul in fp32 (the oracle).
"""
from __future__ import annotations

import torch

from . import _ext

E4M3 = torch.float8_e4m3fn
E4M3_MAX = 448.0


def _pad128(n: int) -> int:
    return (n + 127) // 128 * 128


def _scale(amax: torch.Tensor, pow2: bool) -> torch.Tensor:
    s = amax * (1.0 / E4M3_MAX)
    if pow2:
        # 2^ceil(log2 s): frexp gives s = m 2^e with m in [0.5, 1); m == 0.5 is already a power of two
        m, e = torch.frexp(s)
        s = torch.ldexp(torch.ones_like(s), (e - (m == 0.5).to(e.dtype)).clamp_min(-125))
    return torch.where(amax > 0, s, torch.ones_like(amax))


def quantize_act_torch(x: torch.Tensor, pow2: bool = True):
    M, K = x.shape
    xb = x.float().view(M, K // 128, 128)
    amax = xb.abs().amax(-1)
    scale = _scale(amax, pow2)
    xq = (xb / scale[..., None]).to(E4M3).view(M, K)
    sx = torch.zeros(K // 128, _pad128(M), device=x.device)
    sx[:, :M] = scale.t()
    return xq, sx


def quantize_weight_torch(w: torch.Tensor, pow2: bool = True):
    squeeze = w.dim() == 2
    w3 = w[None] if squeeze else w
    G, N, K = w3.shape
    Np = _pad128(N)
    wp = torch.zeros(G, Np, K, device=w.device, dtype=torch.float32)
    wp[:, :N] = w3.float()
    blocks = wp.view(G, Np // 128, 128, K // 128, 128)
    amax = blocks.abs().amax(dim=(2, 4))
    scale = _scale(amax, pow2)
    q = (blocks / scale[:, :, None, :, None]).to(E4M3).view(G, Np, K)[:, :N]
    return (q[0] if squeeze else q).contiguous(), scale


def dequantize_act(xq: torch.Tensor, sx: torch.Tensor) -> torch.Tensor:
    M, K = xq.shape
    return (xq.float().view(M, K // 128, 128) * sx[:, :M].t()[..., None]).view(M, K)


def dequantize_weight(wq: torch.Tensor, sw: torch.Tensor) -> torch.Tensor:
    squeeze = wq.dim() == 2
    w3 = wq[None] if squeeze else wq
    G, N, K = w3.shape
    s = sw.repeat_interleave(128, dim=1)[:, :N].repeat_interleave(128, dim=2)
    out = w3.float() * s
    return out[0] if squeeze else out


def quantize_act(x: torch.Tensor, pow2: bool = True, offsets: torch.Tensor | None = None):
    """offsets (CUDA, grouped operands): rows at or past offsets[-1] -- read by no GEMM tile --
    are left unwritten."""
    if not _ext.use_cuda(x):
        return quantize_act_torch(x, pow2)
    return tuple(_ext.load().fp8_quant_act(x.contiguous(), pow2, offsets))


def quantize_weight(w: torch.Tensor, pow2: bool = True):
    if not _ext.use_cuda(w):
        return quantize_weight_torch(w, pow2)
    wq, sw = _ext.load().fp8_quant_weight(w.contiguous(), pow2)
    return wq, sw


def fp8_mm(x: torch.Tensor, wq: torch.Tensor, sw: torch.Tensor, scaled_mma: bool = True) -> torch.Tensor:
    """x [M, K] (bf16) @ dequant(wq, sw)^T -> [M, N] bf16, x quantised per 1 x 128 block.
    scaled_mma: sw holds powers of two (quantize_weight's default) and x is quantised the same way."""
    xq, sx = quantize_act(x, pow2=scaled_mma)
    if not _ext.use_cuda(x):
        return (dequantize_act(xq, sx) @ dequantize_weight(wq, sw).t()).to(x.dtype)
    out = torch.empty(x.shape[0], wq.shape[-2], device=x.device, dtype=torch.bfloat16)
    _ext.load().fp8_gemm(xq, sx, wq, sw.reshape(-1), out, scaled_mma=scaled_mma)
    return out


def fp8_grouped_mm(x_perm: torch.Tensor, wq: torch.Tensor, sw: torch.Tensor, offsets: torch.Tensor,
                   rows: int, scaled_mma: bool = True) -> torch.Tensor:
    """Row group g of x_perm (rows [offsets[g], offsets[g+1]), multiples of 128) times
    dequant(wq[g])^T -> [rows, N] bf16."""
    xq, sx = quantize_act(x_perm, pow2=scaled_mma, offsets=offsets if _ext.use_cuda(x_perm) else None)
    if not _ext.use_cuda(x_perm):
        w = dequantize_weight(wq, sw)
        xd = dequantize_act(xq, sx)
        out = torch.zeros(x_perm.shape[0], wq.shape[-2], dtype=torch.float32)
        off = offsets.tolist()
        for g in range(wq.shape[0]):
            out[off[g]:off[g + 1]] = xd[off[g]:off[g + 1]] @ w[g].t()
        return out.to(x_perm.dtype)
    out = torch.empty(x_perm.shape[0], wq.shape[-2], device=x_perm.device, dtype=torch.bfloat16)
    _ext.load().fp8_gemm(xq, sx, wq, sw.reshape(-1), out, offsets, rows, scaled_mma)
    return out


def fp8_grouped_swiglu(x_perm: torch.Tensor, wq: torch.Tensor, sw: torch.Tensor, offsets: torch.Tensor, rows: int,
                       keep_act: bool = True):
    """Expert gate|up GEMM (wq [G, 2F, K], gate / up rows interleaved in groups of 32) with the
    SwiGLU and the 1 x 128 requantisation of silu(g) * u in its epilogue.
    -> (H [rows, 2F] bf16 pre-activation, act [rows, F] bf16 or None, actq [rows, F] e4m3,
        act_scale fp32 [F/128, rows padded to 128]) -- actq / act_scale feed the down GEMM."""
    from .gemm import deinterleave_cols
    F2 = wq.shape[-2]
    if not _ext.use_cuda(x_perm):
        H = fp8_grouped_mm(x_perm, wq, sw, offsets, rows)
        g, u = deinterleave_cols(H.float())
        a = torch.nn.functional.silu(g) * u
        aq, sa = quantize_act_torch(a)
        return H, (a.to(x_perm.dtype) if keep_act else None), aq, sa
    xq, sx = quantize_act(x_perm, offsets=offsets)
    dev = x_perm.device
    R = x_perm.shape[0]
    H = torch.empty(R, F2, device=dev, dtype=torch.bfloat16)
    act = torch.empty(R, F2 // 2, device=dev, dtype=torch.bfloat16) if keep_act else None
    actq = torch.empty(R, F2 // 2, device=dev, dtype=E4M3)
    sa = torch.empty(F2 // 256, _pad128(R), device=dev, dtype=torch.float32)
    _ext.load().fp8_gemm_swiglu_q(xq, sx, wq, sw.reshape(-1), H, act, actq, sa, offsets, rows)
    return H, act, actq, sa


# ----------------------------------------------------------------------------
# training linears: fp8 forward (fprop) and input-gradient (dgrad) GEMMs
# ----------------------------------------------------------------------------
class _WeightCache:
    """Quantised copies of a weight ([N, K] for fprop, [K, N] for dgrad), redone when the
    weight changes: its version counter moves on in-place torch updates, and optimisers that
    write parameters through their own kernels call `bump()` after every step."""

    def __init__(self):
        self._d: dict = {}
        self.generation = 0

    def bump(self):
        self.generation += 1

    def get(self, w: torch.Tensor, transposed: bool):
        import weakref
        key = (id(w), transposed)
        hit = self._d.get(key)
        if hit is not None and hit[0] == (w._version, self.generation) and hit[1]() is w:
            return hit[2]
        src = w.detach().t().contiguous() if transposed else w.detach()
        q = quantize_weight(src.to(torch.bfloat16) if src.is_cuda else src)
        # a weak reference: the cache neither keeps a discarded model's weights alive nor
        # serves a new tensor that reuses a freed one's id; dead entries are dropped here
        self._d = {k: v for k, v in self._d.items() if v[1]() is not None}
        self._d[key] = ((w._version, self.generation), weakref.ref(w), q)
        return q


WEIGHTS = _WeightCache()


def _mm_q(a: torch.Tensor, q) -> torch.Tensor:
    wq, sw = q
    return fp8_mm(a, wq, sw)


class _Fp8LinearFn(torch.autograd.Function):
    @staticmethod
    def forward(ctx, x, w):
        ctx.save_for_backward(x, w)
        return _mm_q(x, WEIGHTS.get(w, False))

    @staticmethod
    def backward(ctx, dy):
        x, w = ctx.saved_tensors
        dy = dy.contiguous()
        dx = _mm_q(dy, WEIGHTS.get(w, True)) if ctx.needs_input_grad[0] else None
        dw = None
        if ctx.needs_input_grad[1]:
            dw = (dy.float().t() @ x.float()).to(w.dtype) if not dy.is_cuda else _wgrad(dy, x)
        return dx, dw


WGRAD_FP8 = True     # weight gradients through the fp8 GEMM (token-dimension 128-blocks) when T % 128 == 0


def quantize_t_torch(x: torch.Tensor):
    """x [T, C] -> (x^T in e4m3 [C, T], fp32 power-of-two scales [T/128, C padded to 256]): one
    scale per column and 128-token block (the operands of a GEMM that reduces over tokens)."""
    T, Cn = x.shape
    xb = x.float().view(T // 128, 128, Cn)
    scale = _scale(xb.abs().amax(1), True)                       # [T/128, C]
    xt = (xb / scale[:, None, :]).to(E4M3).reshape(T, Cn).t().contiguous()
    st = torch.ones(T // 128, (Cn + 255) // 256 * 256, device=x.device)
    st[:, :Cn] = scale
    return xt, st


def wgrad_fp8(dy: torch.Tensor, x: torch.Tensor) -> torch.Tensor:
    """dy^T @ x [N, K] bf16 with both operands quantised per column and 128-token block."""
    C = _ext.load()
    dyt, sdy = C.fp8_quant_t(dy)
    xt, sxt = C.fp8_quant_t(x)
    out = torch.empty(dy.shape[1], x.shape[1], device=dy.device, dtype=torch.bfloat16)
    C.fp8_gemm(dyt, sdy, xt, sxt, out, sw_rows=True)
    return out


def _wgrad(dy: torch.Tensor, x: torch.Tensor) -> torch.Tensor:
    if WGRAD_FP8 and dy.shape[0] % 128 == 0 and dy.shape[1] % 8 == 0 and x.shape[1] % 8 == 0:
        return wgrad_fp8(dy, x)
    from .gemm import mm_tn
    return mm_tn(dy, x)


def fp8_linear(x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    """y = x @ w^T with block-scaled fp8 fprop, dgrad and (token count % 128 == 0) wgrad GEMMs.
    x [T, K], w [N, K]; K and N multiples of 128."""
    shp = x.shape
    y = _Fp8LinearFn.apply(x.reshape(-1, shp[-1]), w)
    return y.view(*shp[:-1], w.shape[0])


class _Fp8SwiGLUFn(torch.autograd.Function):
    """CUDA SwiGLU MLP: fp8 gate|up GEMM whose epilogue applies the SwiGLU and requantises
    silu(g) * u, fp8 down GEMM on that copy; backward: the SwiGLU backward fused into the bf16
    dact GEMM (as in the bf16 MLP), fp8 dgrad through w13, fp8 weight gradients (operands
    quantised per column and 128-token block; bf16 when the token count is not a multiple of 128)."""

    @staticmethod
    def forward(ctx, x, w13, w2):
        C = _ext.load()
        x2 = x.reshape(-1, x.shape[-1]).contiguous()
        T, F2 = x2.shape[0], w13.shape[0]
        xq, sx = quantize_act(x2)
        q13, q2 = WEIGHTS.get(w13, False), WEIGHTS.get(w2, False)
        dev = x.device
        H = torch.empty(T, F2, device=dev, dtype=torch.bfloat16)
        act = torch.empty(T, F2 // 2, device=dev, dtype=torch.bfloat16)
        actq = torch.empty(T, F2 // 2, device=dev, dtype=E4M3)
        sa = torch.empty(F2 // 256, _pad128(T), device=dev, dtype=torch.float32)
        C.fp8_gemm_swiglu_q(xq, sx, q13[0], q13[1].reshape(-1), H, act, actq, sa)
        y = torch.empty(T, w2.shape[0], device=dev, dtype=torch.bfloat16)
        C.fp8_gemm(actq, sa, q2[0], q2[1].reshape(-1), y)
        ctx.save_for_backward(x2, w13, w2, H, act)
        ctx.shape = x.shape
        return y.view(*x.shape[:-1], w2.shape[0])

    @staticmethod
    def backward(ctx, dy):
        from .gemm import EPI_SWIGLU_BWD
        x2, w13, w2, H, act = ctx.saved_tensors
        C = _ext.load()
        dy2 = dy.reshape(-1, dy.shape[-1]).contiguous()
        dw2 = _wgrad(dy2, act)
        dH = torch.empty_like(H)
        C.gemm(dy2, w2, dH, False, True, EPI_SWIGLU_BWD, 1.0, H, None, 256)
        dx = _mm_q(dH, WEIGHTS.get(w13, True)).view(*ctx.shape)
        dw13 = _wgrad(dH, x2)
        return dx, dw13, dw2


def fp8_swiglu_mlp(x: torch.Tensor, w13: torch.Tensor, w2: torch.Tensor) -> torch.Tensor:
    """SwiGLU MLP (w13: gate/up rows interleaved in groups of 32) with fp8 GEMMs; 2F must be a
    multiple of 256 on CUDA (one requantisation block per gate|up tile)."""
    if x.is_cuda and w13.shape[0] % 256 == 0:
        return _Fp8SwiGLUFn.apply(x, w13, w2)
    from .gemm import deinterleave_cols
    h = fp8_linear(x, w13)
    g, u = deinterleave_cols(h)
    act = (torch.nn.functional.silu(g.float()) * u.float()).to(x.dtype)
    return fp8_linear(act, w2)
