"""Rollout-time policy / value forwards on the tcgen05 MLP kernel (csrc/mlp_kernels.cu).

``MlpWeights.from_sequential`` takes the reference's ``nn.Sequential`` stacks
(R/claude_code/model.py ``_mlp`` :34-44 -> ``actor_logits`` / ``critic``) and keeps 16-bit copies
of the Linear weights and fp32 biases on the device.  The 16-bit operand type is bf16 or fp16
(``operand``, one per ``PolicySet``): both run at the same tensor-core rate; fp16's 11-bit
significand keeps logits and log-probs within 1e-3 of the fp32 network (bf16: about 4e-3 of the
largest logit), with activations saturated at +-65504.  ``PolicySet`` registers up to 20 such networks
once (per weight update / pool refresh) and ``forward`` runs any mix of them over row groups:
the main actor + critic on the same rows, or the frozen opponents of a league pool on their
contiguous row blocks, sampling each 21-bin channel with Gumbel-max and summing the log-probs
(the reference's Categorical(logits).sample() / log_prob(.).sum(-1), ppo_gpu.py:273-285).
"""
import ctypes as C

import torch

from . import _lib

HEAD_CATEGORICAL = 1
HEAD_VALUE = 2
OPERANDS = {"bf16": (0, torch.bfloat16), "fp16": (1, torch.float16)}
FP16_MAX = 65504.0
ACTIVATIONS = {"relu": 0, "tanh": 1}


class MlpDesc(C.Structure):
    _fields_ = [("in_dim", C.c_int), ("n_layers", C.c_int), ("width", C.c_int * 4), ("activation", C.c_int),
                ("head", C.c_int), ("act_dim", C.c_int), ("num_bins", C.c_int), ("weight", C.c_void_p * 4),
                ("bias", C.c_void_p * 4), ("operand", C.c_int), ("head_weight_f32", C.c_void_p)]


class PolicyArgs(C.Structure):
    _fields_ = [("x", C.c_void_p), ("rows", C.c_int64), ("ldx", C.c_int64), ("n_groups", C.c_int),
                ("group_end", C.POINTER(C.c_int64)), ("group_net", C.POINTER(C.c_int)), ("nets_per_group", C.c_int),
                ("bins", C.c_void_p), ("bins_stride", C.c_int64), ("bins_offset", C.c_int), ("act_idx", C.c_void_p),
                ("logp", C.c_void_p), ("value", C.c_void_p), ("logits", C.c_void_p), ("logits_ld", C.c_int64),
                ("seed", C.c_uint64), ("step", C.c_uint64), ("deterministic", C.c_int), ("err", C.c_void_p),
                ("cmd", C.c_void_p), ("cmd_stride", C.c_int64), ("cmd_offset", C.c_int), ("grid", C.c_void_p),
                ("step_dev", C.c_void_p), ("group_end_dev", C.c_void_p)]


class MlpWeights:
    """Device 16-bit weights (``operand`` "bf16" or "fp16") + fp32 biases of one Linear stack."""

    def __init__(self, weights, biases, activation="relu", head=HEAD_CATEGORICAL, act_dim=4, num_bins=21,
                 in_width=None, operand="bf16"):
        if operand not in OPERANDS:
            raise ValueError(f"operand must be one of {sorted(OPERANDS)}")
        self.operand = operand
        dt = OPERANDS[operand][1]
        if operand == "fp16":
            big = max(float(w.detach().abs().max()) for w in weights)
            if not big <= FP16_MAX:
                raise ValueError(f"a weight of magnitude {big:.3g} does not fit fp16; use operand='bf16'")
        self.weights = [w.detach().to(dt).contiguous() for w in weights]
        self.biases = [b.detach().to(torch.float32).contiguous() for b in biases]
        # the kernel reads the input in 16-byte units, and all networks of one launch share the
        # input row layout: the first layer gets zero columns up to in_width (default: the next
        # multiple of 8, e.g. 216 for the 214-D external observation), which meet the zero
        # padding of the input rows
        self.obs_dim = self.weights[0].shape[1]
        width = -(-self.obs_dim // 8) * 8 if in_width is None else int(in_width)
        if width < self.obs_dim or width % 8:
            raise ValueError("in_width must be a multiple of 8 not below the network's input width")
        if width != self.obs_dim:
            w0 = self.weights[0]
            pad = torch.zeros(w0.shape[0], width, dtype=w0.dtype, device=w0.device)
            pad[:, :self.obs_dim] = w0
            self.weights[0] = pad
        self.activation = activation
        self.head = head
        self.act_dim, self.num_bins = act_dim, num_bins
        self.in_dim = self.weights[0].shape[1]
        # a value head after a hidden layer runs in fp32 in that layer's epilogue: its weight
        # row is also kept in fp32
        self.head_w32 = (weights[-1].detach().to(device=self.weights[-1].device, dtype=torch.float32).contiguous()
                         if head == HEAD_VALUE and len(self.weights) >= 2 else None)

    @classmethod
    def from_sequential(cls, seq, head, device, act_dim=4, num_bins=21, in_width=None, operand="bf16"):
        linears = [m for m in seq if isinstance(m, torch.nn.Linear)]
        acts = {type(m).__name__.lower() for m in seq if not isinstance(m, torch.nn.Linear)}
        act = "tanh" if "tanh" in acts else "relu"
        if acts - {"tanh", "relu"}:
            raise ValueError(f"unsupported activation(s): {acts}")
        return cls([l.weight.to(device) for l in linears], [l.bias.to(device) for l in linears], act, head,
                   act_dim, num_bins, in_width, operand)

    @torch.no_grad()
    def load_from(self, seq):
        """Copy a same-shaped stack's current parameters into these buffers in place (after an
        optimiser step): the device addresses, hence the registered tensor maps, stay valid."""
        linears = [m for m in seq if isinstance(m, torch.nn.Linear)]
        if len(linears) != len(self.weights):
            raise ValueError("layer count differs from the registered network")
        for w, b, lin in zip(self.weights, self.biases, linears):
            rows, cols = lin.weight.shape
            if w.shape[0] != rows or not (w.shape[1] == cols or (w is self.weights[0] and cols == self.obs_dim)):
                raise ValueError("layer shape differs from the registered network")
            w[:, :cols].copy_(lin.weight)
            b.copy_(lin.bias)
        if self.head_w32 is not None:
            self.head_w32.copy_(linears[-1].weight)

    def desc(self):
        d = MlpDesc()
        d.in_dim = self.in_dim
        d.n_layers = len(self.weights)
        for i, (w, b) in enumerate(zip(self.weights, self.biases)):
            d.width[i] = w.shape[0]
            d.weight[i] = w.data_ptr()
            d.bias[i] = b.data_ptr()
        d.activation = ACTIVATIONS[self.activation]
        d.head = self.head
        d.act_dim, d.num_bins = self.act_dim, self.num_bins
        d.operand = OPERANDS[self.operand][0]
        d.head_weight_f32 = self.head_w32.data_ptr() if self.head_w32 is not None else None
        return d


class PolicySet:
    """A registered group of networks (indices are positions in ``nets``)."""

    def __init__(self, nets):
        self.lib = _lib.load()
        self.nets = list(nets)           # keeps the device buffers alive
        ops = {n.operand for n in self.nets}
        if len(ops) != 1:
            raise ValueError("every network of a policy set must use the same operand type")
        self.operand = ops.pop()
        self.dtype = OPERANDS[self.operand][1]
        arr = (MlpDesc * len(self.nets))(*[n.desc() for n in self.nets])
        handle = C.c_void_p()
        _lib.check(self.lib.f16_mlp_set_create(arr, len(self.nets), C.byref(handle)), "f16_mlp_set_create")
        self.handle = handle
        self.err = torch.zeros(1, dtype=torch.int32, device=self.nets[0].weights[0].device)

    def close(self):
        if self.handle:
            self.lib.f16_mlp_set_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def forward(self, x, groups, nets_per_group=1, bins=None, bins_stride=4, bins_offset=0, act_idx=None,
                logp=None, value=None, logits=None, seed=0, step=0, deterministic=False, cmd=None, cmd_stride=4,
                cmd_offset=0, grid=None, step_dev=None, group_end_dev=None):
        """groups: list of (row_end, [net indices]) with every group starting at a multiple of 128;
        ``x`` is the (rows, ldx) policy input in the set's operand dtype (``self.dtype``).

        ``cmd`` (fp64, optional) receives action_to_env of the sampled bins at
        ``cmd[r * cmd_stride + cmd_offset + c]`` using the fp32 ``grid`` (num_bins values).
        ``step_dev`` (device int64 [1], optional) is added to ``step`` when the kernel runs, so a
        captured CUDA graph draws fresh samples on every replay.  ``group_end_dev`` (device int64
        [len(groups)], optional) supplies the groups' cumulative row ends from device memory, so a
        grouping computed on the device needs no host round trip; the row ends in ``groups`` are
        then ignored (only the network indices are used)."""
        _lib.require_cuda_tensor(x, self.dtype, None, "policy input", None)
        rows, ldx = x.shape[0], x.stride(0)
        if group_end_dev is not None:
            _lib.require_cuda_tensor(group_end_dev, torch.int64, (len(groups),), "group ends", x.device)
        ends = (C.c_int64 * len(groups))(*[0 if group_end_dev is not None else int(g[0]) for g in groups])
        flat = []
        for _, ids in groups:
            ids = list(ids) + [-1] * (nets_per_group - len(ids))
            flat.extend(ids[:nets_per_group])
        netv = (C.c_int * len(flat))(*flat)
        a = PolicyArgs()
        a.x = x.data_ptr(); a.rows = rows; a.ldx = ldx
        a.n_groups = len(groups); a.group_end = ends; a.group_net = netv; a.nets_per_group = nets_per_group
        a.bins = bins.data_ptr() if bins is not None else None
        a.bins_stride = bins_stride; a.bins_offset = bins_offset
        a.act_idx = act_idx.data_ptr() if act_idx is not None else None
        a.logp = logp.data_ptr() if logp is not None else None
        a.value = value.data_ptr() if value is not None else None
        a.logits = logits.data_ptr() if logits is not None else None
        a.logits_ld = logits.stride(0) if logits is not None else 0
        a.seed = seed & (2 ** 64 - 1); a.step = step & (2 ** 64 - 1); a.deterministic = int(bool(deterministic))
        a.err = self.err.data_ptr()
        a.group_end_dev = group_end_dev.data_ptr() if group_end_dev is not None else None
        if step_dev is not None:
            _lib.require_cuda_tensor(step_dev, torch.int64, (1,), "step counter", x.device)
            a.step_dev = step_dev.data_ptr()
        if cmd is not None:
            _lib.require_cuda_tensor(cmd, torch.float64, None, "env commands", x.device)
            _lib.require_cuda_tensor(grid, torch.float32, None, "action grid", x.device)
            a.cmd = cmd.data_ptr(); a.cmd_stride = cmd_stride; a.cmd_offset = cmd_offset
            a.grid = grid.contiguous().data_ptr() if grid.is_contiguous() else None
            if a.grid is None:
                raise ValueError("action grid must be contiguous")
        _lib.check(self.lib.f16_policy_forward(self.handle, C.byref(a), _lib.stream_of(x)), "f16_policy_forward")

    def check_error(self):
        """Host-synchronising check of the kernel's bounded-wait flag."""
        if int(self.err.item()) != 0:
            raise RuntimeError("f16_policy_forward: a bounded pipeline wait timed out")
