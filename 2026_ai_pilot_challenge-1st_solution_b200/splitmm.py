"""fp32-accurate linear layers on the bf16 tensor cores, for the PPO update.

The reference's update (R/cuda_fdm/ppo_gpu.py:2020-2144) multiplies in fp32 (PyTorch's default
matmul precision, which it keeps), so on a B200 its linear layers run as cuBLAS SGEMM on the
CUDA cores.  Here every fp32 operand v is split into three bf16 terms, hi = bf16(v),
lo = bf16(v - hi), mid = bf16(v - hi - lo) (``f16_split3_bf16``; hi + lo + mid carries v's 24
significant bits), and a product A B is assembled from the six term products whose order of
magnitude reaches fp32's unit roundoff -- hi*hi, hi*lo, lo*hi, hi*mid, lo*lo, mid*hi; the three
dropped ones are below 2^-24 relative -- each a bf16 tensor-core GEMM with fp32 accumulation
(``torch.mm(..., out_dtype=torch.float32)``).  Terms that share an operand run as one GEMM over
concatenated K (x's terms are stored side by side: [hi | lo | mid]), so a forward product is
three GEMM calls.  Against fp64 the results stay within 4x of an fp32 SGEMM's error on the
same operands (about 1e-6 relative; TF32 is near 1e-3), at tensor-core speed.

``SplitLinear.apply(x, weight, bias)`` is a drop-in for ``F.linear`` with its own backward
(dx = g W, dW = g^T x, db = sum g, all in the same split arithmetic).
"""
import torch
import torch.nn.functional as F

from . import _lib

_BF = torch.bfloat16
_F32 = torch.float32


def split3(x):
    """(rows, cols) fp32 -> (rows, 3 cols) bf16 [hi | lo | mid]."""
    if x.dim() != 2:
        raise ValueError("split3 takes a 2-D tensor")
    if x.stride(1) != 1 or x.stride(0) % 4 or x.data_ptr() % 16:
        x = x.contiguous()
    rows, cols = x.shape
    out = torch.empty(rows, 3 * cols, dtype=_BF, device=x.device)
    L = _lib.load()
    _lib.check(L.f16_split3_bf16(x.data_ptr(), rows, cols, x.stride(0), out.data_ptr(), 3 * cols,
                                 _lib.stream_of(x)), "f16_split3_bf16")
    return out


def _mm(a, b, acc=None):
    if acc is None:
        return torch.mm(a, b, out_dtype=_F32)
    return torch.addmm(acc, a, b, out_dtype=_F32)


def matmul_nt(xs, ws, k):
    """x W^T from the splits xs = [xh | xl | xm] (M x 3k) and ws = [wh | wl | wm] (N x 3k)."""
    wh, wl, wm = ws[:, :k], ws[:, k:2 * k], ws[:, 2 * k:]
    y = _mm(xs, torch.cat([wh, wh, wh], 1).t())                   # xh wh + xl wh + xm wh
    y = _mm(xs[:, :2 * k], torch.cat([wl, wl], 1).t(), y)         # + xh wl + xl wl
    return _mm(xs[:, :k], wm.t(), y)                              # + xh wm


def matmul_nn(gs, ws, n, k):
    """g W from gs = [gh | gl | gm] (M x 3n) and ws (W = n x k as [wh | wl | wm], n x 3k)."""
    wh, wl, wm = ws[:, :k], ws[:, k:2 * k], ws[:, 2 * k:]
    y = _mm(gs, torch.cat([wh, wh, wh], 0))                       # gh wh + gl wh + gm wh
    y = _mm(gs[:, :2 * n], torch.cat([wl, wl], 0), y)             # + gh wl + gl wl
    return _mm(gs[:, :n], wm, y)                                  # + gh wm


def matmul_tn(gs, xs, n, k):
    """g^T x (n x k) from gs = [gh | gl | gm] (M x 3n) and xs = [xh | xl | xm] (M x 3k)."""
    gh, gl, gm = gs[:, :n], gs[:, n:2 * n], gs[:, 2 * n:]
    t1 = _mm(gh.t(), xs)                                          # [gh xh | gh xl | gh xm]
    t2 = _mm(gl.t(), xs[:, :2 * k])                               # [gl xh | gl xl]
    t3 = _mm(gm.t(), xs[:, :k])                                   # gm xh
    return ((t3 + t2[:, k:]) + (t1[:, 2 * k:] + t2[:, :k])) + (t1[:, k:2 * k] + t1[:, :k])


class SplitLinear(torch.autograd.Function):
    """F.linear(x, weight, bias) with fp32-accurate tensor-core products (module docstring)."""

    @staticmethod
    def forward(ctx, x, weight, bias):
        k = x.shape[1]
        ws = split3(weight.detach())
        y = matmul_nt(split3(x.detach()), ws, k)
        if bias is not None:
            y = y + bias
        ctx.save_for_backward(x, weight)
        ctx.has_bias = bias is not None
        return y

    @staticmethod
    def backward(ctx, g):
        x, weight = ctx.saved_tensors
        n, k = weight.shape
        g = g.contiguous()
        gs = split3(g)
        gx = gw = gb = None
        if ctx.needs_input_grad[0]:
            gx = matmul_nn(gs, split3(weight), n, k)
        if ctx.needs_input_grad[1]:
            gw = matmul_tn(gs, split3(x), n, k)
        if ctx.has_bias and ctx.needs_input_grad[2]:
            gb = g.sum(0)
        return gx, gw, gb


def usable(layer, x):
    """Whether a linear layer's product can take the split path (CUDA fp32, dims in 16-byte
    units and wide enough to be worth it); other layers stay plain fp32."""
    return (x.is_cuda and x.dtype == _F32 and x.dim() == 2 and layer.in_features % 8 == 0
            and layer.out_features % 8 == 0 and layer.in_features >= 64 and layer.out_features >= 64)


def linear(layer, x):
    """layer(x) for an nn.Linear, through SplitLinear when `usable`."""
    if usable(layer, x):
        return SplitLinear.apply(x, layer.weight, layer.bias)
    return F.linear(x, layer.weight, layer.bias)
