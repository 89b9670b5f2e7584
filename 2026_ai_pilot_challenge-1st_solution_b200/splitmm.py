"""fp32-accurate linear layers on the bf16 tensor cores, for the PPO update.

The reference's update (R/cuda_fdm/ppo_gpu.py:2020-2144) multiplies in fp32 (PyTorch's default
matmul precision, which it keeps), so on a B200 its linear layers run as cuBLAS SGEMM on the
CUDA cores.  Here every fp32 operand v is split into three bf16 terms, hi = bf16(v),
lo = bf16(v - hi), mid = bf16(v - hi - lo) (hi + lo + mid carries v's 24 significant bits),
stored as a row of three parts [mid | lo | hi], and a product A B is assembled from the six term
products whose order of magnitude reaches fp32's unit roundoff -- hi*hi, hi*lo, lo*hi, hi*mid,
lo*lo, mid*hi; the three dropped ones are below 2^-24 relative -- each a bf16 tensor-core GEMM
with fp32 accumulation (``torch.mm(..., out_dtype=torch.float32)``).  Terms that share an
operand run as one GEMM over concatenated K, so a product is three GEMM calls -- or one, when the
producer of the big operand writes it as six parts [mid | lo | hi | lo | hi | hi] against
B = [hi; hi; mid; lo; lo; hi] (``parts_for`` picks the layout that moves fewer bytes).

Accuracy depends on the order: the tensor cores' fp32 accumulation loses more per addition than
an SGEMM's round-to-nearest FMA chain, so the number of additions made at the full magnitude of
the result is kept small.  The five small terms accumulate first (at 2^-8 of the result's
magnitude, where their rounding is negligible), and hi*hi comes last: as the last K range of the
single GEMM, or as a GEMM of its own whose result joins them in cuBLAS's fp32 epilogue (beta = 1,
in place).  A weight gradient reduces
over all rows of a minibatch, so its hi*hi product is a batched GEMM over ``ROW_CHUNK``-row
slices whose partial products are summed in fp32.  Against fp64 the products stay within a few
times an SGEMM's error on the same operands (about 1e-6 relative; TF32 is near 1e-3).

``run_tower(seq, x)`` runs a Linear/activation ``nn.Sequential`` as ``SplitBlock`` autograd
functions: per layer the products, then one kernel for bias + activation that also writes the
split the next layer reads (``f16_bias_act_split``); backward one kernel for the activation
derivative, the split of the gradient and the bias-gradient partial sums
(``f16_act_grad_split``), then the input- and weight-gradient products.  A last hidden layer
followed by a width-1 Linear (the critic's value head) runs as ``SplitValueBlock``: the head's
dot product joins the epilogue kernel (``f16_bias_act_value``) and its backward the prologue
kernel (``f16_act_grad_split_value``).
"""
import torch
import torch.nn as nn
import torch.nn.functional as F

from . import _lib

_BF = torch.bfloat16
_F32 = torch.float32

ACT_NONE, ACT_RELU, ACT_TANH = 0, 1, 2
_ACT_CODES = {nn.ReLU: ACT_RELU, nn.Tanh: ACT_TANH}
ROW_CHUNK = 1024            # rows per tensor-core reduction of a weight gradient's hi*hi term
GRAD_BLOCKS = 148 * 8       # blocks (bias-gradient partial rows) of f16_act_grad_split
MAX_COLS = 1024             # widest layer output f16_act_grad_split takes


def part_width(cols):
    """Column count of one split part: `cols` rounded up to 8 (16 bytes of bf16)."""
    return (cols + 7) & ~7


def _fp32_operand(x):
    if x.stride(1) != 1 or x.stride(0) % 4 or x.data_ptr() % 16:
        x = x.contiguous()
    return x


def parts_for(out_cols, part):
    """Split layout of a product's A operand (`part` columns per term) whose result has `out_cols`
    columns: six parts -- one GEMM -- when the two read-modify-write passes over the fp32 result it
    saves (16 bytes per output column and row) outweigh the three extra parts written (6 bytes
    per column and row), else three parts and three GEMMs."""
    return 6 if 16 * out_cols > 6 * part else 3


def split3(x, parts=3):
    """(rows, cols) fp32 -> (rows, parts p) bf16 [mid | lo | hi] (+ [lo | hi | hi] for six parts),
    p = part_width(cols), pad columns zero (cols must be a multiple of 4)."""
    if x.dim() != 2:
        raise ValueError("split3 takes a 2-D tensor")
    x = _fp32_operand(x)
    rows, cols = x.shape
    p = part_width(cols)
    out = torch.empty(rows, parts * p, dtype=_BF, device=x.device)
    _lib.check(_lib.load().f16_split3_bf16(x.data_ptr(), rows, cols, x.stride(0), out.data_ptr(), parts * p, parts,
                                           _lib.stream_of(x)), "f16_split3_bf16")
    return out


def bias_act_split(y, bias, act, parts):
    """y := act(y + bias) in place (y a fresh fp32 product); returns the split of the result in
    `parts` parts (3 or 6), or None for parts 0."""
    rows, cols = y.shape
    hs = torch.empty(rows, parts * part_width(cols), dtype=_BF, device=y.device) if parts else None
    bias = bias.detach().contiguous()
    _lib.check(_lib.load().f16_bias_act_split(y.data_ptr(), rows, cols, y.stride(0), bias.data_ptr(), act,
                                              hs.data_ptr() if hs is not None else None,
                                              hs.stride(0) if hs is not None else 0, parts if parts else 3,
                                              _lib.stream_of(y)), "f16_bias_act_split")
    return hs


def act_grad_split(gh, h, act, parts=3):
    """(split of g_y in `parts` parts, bias gradient) for g_y = act'(gh; h)."""
    gh = _fp32_operand(gh)
    rows, cols = gh.shape
    nblk = max(1, min(GRAD_BLOCKS, (rows + 63) // 64))
    gys = torch.empty(rows, parts * part_width(cols), dtype=_BF, device=gh.device)
    part = torch.empty(nblk, cols, dtype=_F32, device=gh.device)
    _lib.check(_lib.load().f16_act_grad_split(gh.data_ptr(), gh.stride(0), h.data_ptr(), h.stride(0), rows, cols, act,
                                              gys.data_ptr(), gys.stride(0), parts, part.data_ptr(), nblk,
                                              _lib.stream_of(gh)), "f16_act_grad_split")
    return gys, part.sum(0)


def bias_act_value(y, bias, act, wv, bv):
    """y := act(y + bias) in place; returns v = y wv + bv (M,) (wv, bv device tensors)."""
    rows, cols = y.shape
    v = torch.empty(rows, dtype=_F32, device=y.device)
    _lib.check(_lib.load().f16_bias_act_value(y.data_ptr(), rows, cols, y.stride(0), bias.detach().contiguous().data_ptr(),
                                              act, wv.data_ptr(), bv.data_ptr(), v.data_ptr(), _lib.stream_of(y)),
               "f16_bias_act_value")
    return v


def act_grad_split_value(gv, wv, h, act, parts=3):
    """(split of g_y in `parts` parts, bias gradient, value-weight gradient) for
    g_y = act'(gv wv^T; h)."""
    rows, cols = h.shape
    nblk = max(1, min(GRAD_BLOCKS, (rows + 63) // 64))
    gys = torch.empty(rows, parts * part_width(cols), dtype=_BF, device=h.device)
    part = torch.empty(nblk, cols, dtype=_F32, device=h.device)
    vpart = torch.empty(nblk, cols, dtype=_F32, device=h.device)
    _lib.check(_lib.load().f16_act_grad_split_value(gv.data_ptr(), wv.data_ptr(), h.data_ptr(), h.stride(0), rows,
                                                    cols, act, gys.data_ptr(), gys.stride(0), parts, part.data_ptr(),
                                                    vpart.data_ptr(), nblk, _lib.stream_of(h)),
               "f16_act_grad_split_value")
    return gys, part.sum(0), vpart.sum(0)


def _mm(a, b, acc=None):
    """a b in fp32 (bf16 operands, fp32 accumulation); with `acc`, added into it in place."""
    if acc is None:
        return torch.mm(a, b, out_dtype=_F32)
    return torch.addmm(acc, a, b, out_dtype=_F32, out=acc)


def _parts(s, p):
    """(mid, lo, hi) views of a split."""
    return s[:, :p], s[:, p:2 * p], s[:, 2 * p:3 * p]


def matmul_nt(xs, ws, k):
    """x W^T from the splits xs (M x 3k or 6k) and ws (N x 3k); k a multiple of 8."""
    wm, wl, wh = _parts(ws, k)
    if xs.shape[1] == 6 * k:                                      # [xm | xl | xh | xl | xh | xh]
        return _mm(xs, torch.cat([wh, wh, wm, wl, wl, wh], 1).t())
    y = _mm(xs[:, :3 * k], torch.cat([wh, wh, wm], 1).t())        # xm wh + xl wh + xh wm
    y = _mm(xs[:, k:3 * k], torch.cat([wl, wl], 1).t(), y)        # + xl wl + xh wl
    return _mm(xs[:, 2 * k:3 * k], wh.t(), y)                     # + xh wh


def matmul_nn(gs, ws, n, k):
    """g W from gs (M x 3p or 6p, p = part_width(n)) and ws (W = n x k, split n x 3k); W's terms
    get p - n zero rows against g's zero pad columns."""
    p = part_width(n)
    wm, wl, wh = _parts(ws, k)
    if p != n:
        pad = ws.new_zeros(p - n, k)
        wm, wl, wh = (torch.cat([t, pad], 0) for t in (wm, wl, wh))
    if gs.shape[1] == 6 * p:                                      # [gm | gl | gh | gl | gh | gh]
        return _mm(gs, torch.cat([wh, wh, wm, wl, wl, wh], 0))
    y = _mm(gs[:, :3 * p], torch.cat([wh, wh, wm], 0))            # gm wh + gl wh + gh wm
    y = _mm(gs[:, p:3 * p], torch.cat([wl, wl], 0), y)            # + gl wl + gh wl
    return _mm(gs[:, 2 * p:3 * p], wh, y)                         # + gh wh


def _tn_chunked(a, b):
    """a^T b over M rows (a: M x p, b: M x k views) as ROW_CHUNK-row tensor-core products whose
    (p x k) partials are summed in fp32."""
    m = a.shape[0]
    c = m // ROW_CHUNK
    if c < 2:
        return _mm(a.t(), b)
    m0 = c * ROW_CHUNK
    out = torch.bmm(a[:m0].unflatten(0, (c, ROW_CHUNK)).transpose(1, 2), b[:m0].unflatten(0, (c, ROW_CHUNK)),
                    out_dtype=_F32).sum(0)
    if m0 < m:
        out += _mm(a[m0:].t(), b[m0:])
    return out


def matmul_tn(gs, xs, n, k):
    """g^T x (n x k) from gs (p = part_width(n) per part) and xs (k per part), three or six parts
    each (only the first three are read)."""
    gm, gl, gh = _parts(gs, part_width(n))
    xh = xs[:, 2 * k:3 * k]
    a = _mm(gh.t(), xs[:, :2 * k])                                # [gh xm | gh xl]
    b = _mm(gl.t(), xs[:, k:3 * k])                               # [gl xl | gl xh]
    c = _mm(gm.t(), xh)                                           # gm xh
    small = ((c + b[:, :k]) + a[:, :k]) + (a[:, k:] + b[:, k:])
    return (_tn_chunked(gh, xh) + small)[:n]


def _grad_parts(ctx, n, k):
    """Layout of a layer's output-gradient split: six parts when the input gradient g W (k
    columns) is computed and gains by it, else three (the weight gradient reads three)."""
    return parts_for(k, part_width(n)) if ctx.needs_input_grad[0] else 3


class SplitBlock(torch.autograd.Function):
    """h = act(x W^T + b) with fp32-accurate tensor-core products (module docstring).

    Inputs: x (fp32, for the autograd graph), xs = split3(x) (the operand actually read), the
    layer's weight and bias, the activation code and the part count (0, 3 or 6) of the split of
    h to return.  Returns (h, hs); hs is empty when not requested and never carries a gradient."""

    @staticmethod
    def forward(ctx, x, xs, weight, bias, act, out_parts):
        ctx.set_materialize_grads(False)
        n, k = weight.shape
        ws = split3(weight.detach())
        p = part_width(n)
        if p != n:
            # a width off the 16-byte grid (the 84 logits): multiply by p - n extra zero rows so
            # the product's rows stay aligned, and return the first n columns
            ws = torch.cat([ws, ws.new_zeros(p - n, ws.shape[1])], 0)
        y = matmul_nt(xs, ws, k)
        if p != n:
            y = y[:, :n]
        hs = bias_act_split(y, bias, act, out_parts)
        if hs is None:
            hs = y.new_empty(0, dtype=_BF)
        ctx.mark_non_differentiable(hs)
        ctx.act = act
        ctx.save_for_backward(xs, weight, y)          # y now holds h
        return y, hs

    @staticmethod
    def backward(ctx, gh, _ghs):
        if gh is None:
            return None, None, None, None, None, None
        xs, weight, h = ctx.saved_tensors
        n, k = weight.shape
        gys, gb = act_grad_split(gh, h, ctx.act, _grad_parts(ctx, n, k))
        gx = matmul_nn(gys, split3(weight.detach()), n, k) if ctx.needs_input_grad[0] else None
        gw = matmul_tn(gys, xs, n, k) if ctx.needs_input_grad[2] else None
        return gx, None, gw, (gb if ctx.needs_input_grad[3] else None), None, None


class SplitValueBlock(torch.autograd.Function):
    """v = act(x W^T + b) wv^T + bv: a SplitBlock whose output feeds a width-1 Linear (the
    critic's value head), the head folded into the layer's epilogue and backward prologue.
    Returns v as (M, 1) like the Linear it replaces."""

    @staticmethod
    def forward(ctx, x, xs, weight, bias, act, wv, bv):
        ctx.set_materialize_grads(False)
        k = weight.shape[1]
        y = matmul_nt(xs, split3(weight.detach()), k)
        v = bias_act_value(y, bias, act, wv.detach().reshape(-1).contiguous(), bv.detach().reshape(-1).contiguous())
        ctx.act = act
        ctx.save_for_backward(xs, weight, y, wv)      # y now holds h
        return v.unsqueeze(1)

    @staticmethod
    def backward(ctx, gvo):
        if gvo is None:
            return None, None, None, None, None, None, None
        xs, weight, h, wv = ctx.saved_tensors
        n, k = weight.shape
        gv = gvo.reshape(-1).contiguous()
        gys, gb, gwv = act_grad_split_value(gv, wv.detach().reshape(-1).contiguous(), h, ctx.act,
                                            _grad_parts(ctx, n, k))
        need = ctx.needs_input_grad
        gx = matmul_nn(gys, split3(weight.detach()), n, k) if need[0] else None
        gw = matmul_tn(gys, xs, n, k) if need[2] else None
        return (gx, None, gw, gb if need[3] else None, None, gwv.view(1, n) if need[5] else None,
                gv.sum().reshape(1) if need[6] else None)


def _dims_ok(layer):
    return (layer.in_features % 8 == 0 and layer.out_features % 4 == 0 and layer.in_features >= 64
            and 64 <= layer.out_features <= MAX_COLS)


def usable(layer, x):
    """Whether a linear layer's product can take the split path (CUDA fp32 input, input width in
    16-byte units, output width a multiple of 4 -- padded to 8 inside -- and both wide enough to
    be worth it); other layers stay plain fp32."""
    return x.is_cuda and x.dtype == _F32 and x.dim() == 2 and _dims_ok(layer)


def _in_parts(layer):
    return parts_for(layer.out_features, part_width(layer.in_features))


SHARE_SPLIT = "_f16_share_split"     # set True on an input tensor to keep its split for reuse


def _input_split(x, parts):
    """split3(x, parts) for a tower's input.  An input marked with SHARE_SPLIT (the trainer marks
    each minibatch's observations) keeps its split on the tensor, so a second tower on the same
    input (the critic after the actor) reuses it; the tensor's version counter invalidates it if
    x is modified in place.  Unmarked inputs keep nothing (no memory held past the call)."""
    if not getattr(x, SHARE_SPLIT, False):
        return split3(x.detach(), parts)
    cached = getattr(x, "_f16_split", None)
    if cached is not None and cached[0] == parts and cached[1] == x._version:
        return cached[2]
    xs = split3(x.detach(), parts)
    try:
        x._f16_split = (parts, x._version, xs)
    except (AttributeError, RuntimeError):
        pass
    return xs


def split_linear(x, weight, bias, act=ACT_NONE):
    """act(F.linear(x, weight, bias)) through one SplitBlock."""
    xs = split3(x.detach(), parts_for(weight.shape[0], part_width(weight.shape[1])))
    return SplitBlock.apply(x, xs, weight, bias, act, 0)[0]


def run_tower(seq, x):
    """seq(x) for a Sequential of Linear and ReLU/Tanh modules: each Linear (+ the activation
    that follows it) the split path takes runs as a SplitBlock, the others as plain fp32 torch."""
    mods = list(seq)
    xs = None
    i = 0
    while i < len(mods):
        m = mods[i]
        if not isinstance(m, nn.Linear):
            x, xs = m(x), None
            i += 1
            continue
        act_mod = mods[i + 1] if i + 1 < len(mods) and not isinstance(mods[i + 1], nn.Linear) else None
        code = ACT_NONE if act_mod is None else _ACT_CODES.get(type(act_mod))
        if code is None or not usable(m, x):
            x, xs = F.linear(x, m.weight, m.bias), None
            i += 1
            continue
        if xs is None:
            xs = _input_split(x, _in_parts(m))
        head = mods[i + 2] if act_mod is not None and i + 3 == len(mods) else None
        if (isinstance(head, nn.Linear) and head.out_features == 1 and head.in_features == m.out_features
                and m.out_features % 8 == 0 and head.bias is not None):
            return SplitValueBlock.apply(x, xs, m.weight, m.bias, code, head.weight, head.bias)
        step = 1 if act_mod is None else 2
        nxt = mods[i + step] if i + step < len(mods) else None
        out_parts = _in_parts(nxt) if isinstance(nxt, nn.Linear) and _dims_ok(nxt) else 0
        x, hs = SplitBlock.apply(x, xs, m.weight, m.bias, code, out_parts)
        xs = hs if out_parts else None
        i += step
    return x
