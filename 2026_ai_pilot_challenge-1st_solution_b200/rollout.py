"""Rollout arithmetic of the reference trainer on the sm_100a kernels (R/cuda_fdm/ppo_gpu.py).

* ``RunningNorm``      -- drop-in for ppo_gpu.RunningNorm (:184-222): same attributes
  (mean, var, count fp32 tensors, clip, eps) and methods (update, normalize, state_dict,
  load_state_dict, clone); update / normalize run f16_norm_update / f16_norm_apply, and
  ``normalize_half`` (``normalize_bf16``) also emits the zero-padded 16-bit matrix (bf16 or fp16,
  the policy set's operand type) the MLP kernel consumes.
* ``gae``              -- the GAE loop of collect_rollout (:1983-1995) in one launch, bit-exact.
* ``make_action_grid`` / ``action_to_env`` -- the reference action mapping (:178-180, :361-369).
"""
import torch

from . import _lib


def make_action_grid(num_bins=21, device="cpu"):
    return torch.linspace(-1.0, 1.0, int(num_bins), device=device)


def action_to_env(idx, num_bins, grid=None):
    """Action indices (N,4) -> env controls (N,4): grid value, throttle 0.5*v + 0.5."""
    if grid is None:
        grid = make_action_grid(num_bins, device=idx.device)
    cont = grid[idx.long()]
    ctrl = cont.clone()
    ctrl[:, 3] = 0.5 * cont[:, 3] + 0.5
    return ctrl


class RunningNorm:
    def __init__(self, dim, device, clip=10.0, eps=1e-8):
        self.dim = int(dim)
        self.device = torch.device(device)
        if self.device.type == "cuda" and self.device.index is None:
            self.device = torch.device("cuda", torch.cuda.current_device())
        self.mean = torch.zeros(dim, device=self.device, dtype=torch.float32)
        self.var = torch.ones(dim, device=self.device, dtype=torch.float32)
        self.count = torch.zeros((), device=self.device, dtype=torch.float32) + 1e-4
        self.clip = float(clip)
        self.eps = float(eps)
        self._scratch = None
        self.lib = _lib.load()

    def _x(self, x):
        _lib.require_cuda_tensor(x, torch.float32, None, "observations", self.device)
        if x.dim() != 2 or x.shape[1] != self.dim:
            raise ValueError(f"observations must be (B, {self.dim})")
        return x if x.stride(1) == 1 else x.contiguous()

    @torch.no_grad()
    def update(self, x, group=None):
        """Merge the batch x into the running statistics.  With a torch.distributed ``group`` of
        more than one rank the batch is the union of every rank's x (per-feature fp64 sums are
        all-reduced before the merge; every rank must pass the same number of rows), so all ranks
        keep the same normaliser."""
        x = self._x(x)
        B = x.shape[0]
        need = int(self.lib.f16_norm_scratch_doubles(B, self.dim))
        if self._scratch is None or self._scratch.numel() < need:
            self._scratch = torch.empty(need, dtype=torch.float64, device=self.device)
        stream = _lib.stream_of(x)
        world = 1
        if group is not None:
            import torch.distributed as dist
            world = dist.get_world_size(group)
        if world == 1:
            _lib.check(self.lib.f16_norm_update(_lib.ptr(x), B, self.dim, x.stride(0), _lib.ptr(self.mean),
                                                _lib.ptr(self.var), _lib.ptr(self.count), _lib.ptr(self._scratch),
                                                self._scratch.numel(), stream), "f16_norm_update")
            return
        import torch.distributed as dist
        sums = torch.empty(self.dim * 2, dtype=torch.float64, device=self.device)
        _lib.check(self.lib.f16_norm_sums(_lib.ptr(x), B, self.dim, x.stride(0), _lib.ptr(sums),
                                          _lib.ptr(self._scratch), self._scratch.numel(), stream), "f16_norm_sums")
        dist.all_reduce(sums, group=group)
        total = B * world                       # every rank holds the same number of environments
        _lib.check(self.lib.f16_norm_merge_sums(_lib.ptr(sums), total, self.dim, _lib.ptr(self.mean),
                                                _lib.ptr(self.var), _lib.ptr(self.count), stream),
                   "f16_norm_merge_sums")

    @torch.no_grad()
    def normalize(self, x, out=None):
        x = self._x(x)
        y = torch.empty_like(x) if out is None else out
        _lib.check(self.lib.f16_norm_apply(_lib.ptr(x), x.shape[0], self.dim, x.stride(0), _lib.ptr(self.mean),
                                           _lib.ptr(self.var), self.eps, self.clip, _lib.ptr(y), y.stride(0), None,
                                           0, _lib.stream_of(x)), "f16_norm_apply")
        return y

    @torch.no_grad()
    def normalize_half(self, x, out_f32=None, out_half=None, pad_to=192, nonfinite=None, dtype=torch.bfloat16):
        """Normalised rows as fp32 (optional) and as a (B, pad_to) zero-padded 16-bit matrix
        (``out_half``'s dtype, else ``dtype``: bf16 or fp16); ``nonfinite`` (a device uint32/int32
        counter, optional) is incremented when an output value is NaN or infinite."""
        x = self._x(x)
        yh = torch.empty(x.shape[0], pad_to, dtype=dtype, device=x.device) if out_half is None else out_half
        _lib.check(self.lib.f16_norm_apply_half(
            _lib.ptr(x), x.shape[0], self.dim, x.stride(0), _lib.ptr(self.mean), _lib.ptr(self.var), self.eps,
            self.clip, _lib.ptr(out_f32) if out_f32 is not None else None,
            out_f32.stride(0) if out_f32 is not None else 0, _lib.ptr(yh), yh.stride(0), half_operand(yh),
            _lib.ptr(nonfinite) if nonfinite is not None else None, _lib.stream_of(x)), "f16_norm_apply_half")
        return yh

    def normalize_bf16(self, x, out_f32=None, out_bf16=None, pad_to=192, nonfinite=None):
        """normalize_half with a bf16 output."""
        if out_bf16 is not None and out_bf16.dtype != torch.bfloat16:
            raise TypeError("normalize_bf16 writes a bf16 matrix")
        return self.normalize_half(x, out_f32, out_bf16, pad_to, nonfinite, torch.bfloat16)

    def state_dict(self):
        return {"mean": self.mean.clone(), "var": self.var.clone(), "count": self.count.clone()}

    def load_state_dict(self, sd):
        self.mean.copy_(sd["mean"]); self.var.copy_(sd["var"]); self.count.copy_(sd["count"])

    def clone(self):
        c = RunningNorm(self.dim, self.device, self.clip, self.eps)
        c.load_state_dict(self.state_dict())
        return c


def half_operand(t):
    """C-ABI operand code of a 16-bit policy-input tensor (bf16 0, fp16 1)."""
    if t.dtype == torch.bfloat16:
        return 0
    if t.dtype == torch.float16:
        return 1
    raise TypeError(f"policy input must be bf16 or fp16, got {t.dtype}")


@torch.no_grad()
def cast_half(x, out_half, out_f32=None, nonfinite=None):
    """Un-normalised rows (B, D) fp32 into a zero-padded (B, ldb) 16-bit policy input (bf16 or
    fp16, ``out_half``'s dtype; and optionally an fp32 copy) in one kernel: the input of a
    network without a normaliser."""
    _lib.require_cuda_tensor(x, torch.float32, None, "observations", None)
    if x.dim() != 2 or x.stride(1) != 1:
        raise ValueError("observations must be (B, D) with unit column stride")
    L = _lib.load()
    _lib.check(L.f16_norm_apply_half(_lib.ptr(x), x.shape[0], x.shape[1], x.stride(0), None, None, 0.0, 0.0,
                                     _lib.ptr(out_f32) if out_f32 is not None else None,
                                     out_f32.stride(0) if out_f32 is not None else 0, _lib.ptr(out_half),
                                     out_half.stride(0), half_operand(out_half),
                                     _lib.ptr(nonfinite) if nonfinite is not None else None,
                                     _lib.stream_of(x)), "f16_norm_apply_half")
    return out_half


cast_bf16 = cast_half


def gae(b_rew, b_val, b_done, last_value, next_done, gamma, gae_lambda, adv=None, ret=None):
    """(adv, ret) of collect_rollout's GAE; all (T, nenv) / (nenv,) fp32 CUDA tensors."""
    T, n = b_rew.shape
    dev = b_rew.device
    for t, name in ((b_rew, "rewards"), (b_val, "values"), (b_done, "dones")):
        _lib.require_cuda_tensor(t, torch.float32, (T, n), name, dev)
    for t, name in ((last_value, "last value"), (next_done, "next done")):
        _lib.require_cuda_tensor(t, torch.float32, (n,), name, dev)
    tens = [x.contiguous() for x in (b_rew, b_val, b_done, last_value, next_done)]
    adv = torch.empty_like(tens[0]) if adv is None else adv
    ret = torch.empty_like(tens[0]) if ret is None else ret
    L = _lib.load()
    _lib.check(L.f16_gae(*[_lib.ptr(x) for x in tens], T, n, n, float(gamma), float(gae_lambda), _lib.ptr(adv),
                         _lib.ptr(ret), _lib.stream_of(adv)), "f16_gae")
    return adv, ret
