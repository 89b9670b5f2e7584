"""The PPO update's categorical head on the sm_100a kernels.

``MLPDiscreteActorCritic.evaluate_actions`` (R/claude_code/model.py:198-215) builds
``torch.distributions.Categorical(logits=z.view(-1, A, B))`` and returns
``log_prob(action).sum(-1)`` and ``entropy().sum(-1)``: about a dozen torch kernels over the
(M, A, B) logits forward and as many backward.  ``logp_entropy`` computes the same two vectors in
one kernel (``f16_categorical_fwd``) and their gradient with respect to the logits in one more
(``f16_categorical_bwd``), with torch's formulation (logsumexp-normalised logits, softmax of
those, entropy over logits clamped at -FLT_MAX).  The distribution's argument checks are kept:
a NaN logit or an action outside [0, B) raises ValueError as torch's validation does (one host
read of the kernel's flag word, where torch reads its two checks).
"""
import torch

from . import _lib

MAX_BINS = 32
MAX_WIDTH = 128


class _Head(torch.autograd.Function):
    @staticmethod
    def forward(ctx, logits, action, act_dim, num_bins, flags):
        ctx.set_materialize_grads(False)
        m = logits.shape[0]
        logp = torch.empty(m, dtype=torch.float32, device=logits.device)
        ent = torch.empty(m, dtype=torch.float32, device=logits.device)
        _lib.check(_lib.load().f16_categorical_fwd(logits.data_ptr(), logits.stride(0), m, act_dim, num_bins,
                                                   action.data_ptr(), action.element_size(), logp.data_ptr(),
                                                   ent.data_ptr(), flags.data_ptr(), _lib.stream_of(logits)),
                   "f16_categorical_fwd")
        ctx.save_for_backward(logits, action)
        ctx.dims = (act_dim, num_bins)
        return logp, ent

    @staticmethod
    def backward(ctx, g_lp, g_ent):
        logits, action = ctx.saved_tensors
        if g_lp is None and g_ent is None:
            return None, None, None, None, None
        act_dim, num_bins = ctx.dims
        m = logits.shape[0]
        gz = torch.empty(m, act_dim * num_bins, dtype=torch.float32, device=logits.device)
        g_lp = g_lp.contiguous() if g_lp is not None else None
        g_ent = g_ent.contiguous() if g_ent is not None else None
        _lib.check(_lib.load().f16_categorical_bwd(logits.data_ptr(), logits.stride(0), m, act_dim, num_bins,
                                                   action.data_ptr(), action.element_size(), _lib.ptr(g_lp),
                                                   _lib.ptr(g_ent), gz.data_ptr(), gz.stride(0),
                                                   _lib.stream_of(logits)), "f16_categorical_bwd")
        return gz, None, None, None, None


def usable(logits, act_dim, num_bins):
    return (logits.is_cuda and logits.dtype == torch.float32 and logits.dim() == 2 and logits.stride(1) == 1
            and logits.shape[1] == act_dim * num_bins and num_bins <= MAX_BINS and act_dim * num_bins <= MAX_WIDTH)


def logp_entropy(logits, action, act_dim, num_bins):
    """(sum over the A groups of log_prob(action), sum of the entropies) for logits (M, A*B) and
    action (M, A) category indices (uint8 as is, other dtypes through .long() as the reference)."""
    m = logits.shape[0]
    action = action.reshape(m, act_dim)
    action = action.contiguous() if action.dtype == torch.uint8 else action.long().contiguous()
    flags = torch.zeros(1, dtype=torch.int32, device=logits.device)
    logp, ent = _Head.apply(logits, action, act_dim, num_bins, flags)
    bad = int(flags.item())
    if bad & 1:
        raise ValueError(f"Expected parameter logits (Tensor of shape ({m}, {act_dim}, {num_bins})) of distribution "
                         "Categorical to satisfy the constraint IndependentConstraint(Real(), 1), but found invalid "
                         "values")
    if bad & 2:
        raise ValueError(f"Expected value argument (Tensor of shape ({m}, {act_dim})) to be within the support "
                         f"(IntegerInterval(lower_bound=0, upper_bound={num_bins - 1})) of the distribution "
                         "Categorical, but found invalid values")
    return logp, ent
