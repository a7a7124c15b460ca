"""CPU stand-ins for the per-shard CUDA kernels used by kbb200.dist, so the
sharding and collective composition can run on gloo ranks without a GPU.
They follow the C-ABI contracts: fp64 partials, fp32 outputs."""
from __future__ import annotations

import math

import torch


def mse_partial(a, b):
    """[sum((a - b)^2), element count], fp64."""
    d = a.double() - b.double()
    return torch.stack([(d * d).sum(), torch.tensor(float(a.numel()), dtype=torch.float64)])


def mse_finalize(total, total_n=0, out=None):
    r = (total[0] / (total_n if total_n > 0 else total[1])).float()
    if out is not None:
        out.copy_(r)
        return out
    return r


def sumsq_partial(x):
    return (x.double() ** 2).sum().reshape(())


def scale_by_inv_norm(x, total, out=None):
    norm = torch.sqrt(total).float()
    r = x / norm
    if out is not None:
        out.copy_(r)
        return out
    return r


def batch_norm_stats(x):
    """[sums (C), sums of squares (C), elements per channel], fp64."""
    axes = [0] + list(range(2, x.dim()))
    xd = x.double()
    count = x.shape[0] * math.prod(x.shape[2:])
    return torch.cat([xd.sum(axes), (xd * xd).sum(axes), torch.tensor([float(count)], dtype=torch.float64)])


def batch_norm_apply(x, stats, count, weight, bias, eps, momentum, running_mean, running_var, out=None):
    C = x.shape[1]
    count = count if count > 0 else float(stats[2 * C])
    mean = stats[:C] / count
    var = (stats[C:2 * C] / count - mean * mean).clamp_min(0)
    shape = [1, -1] + [1] * (x.dim() - 2)
    y = (x.double() - mean.reshape(shape)) / torch.sqrt(var + eps).reshape(shape)
    if weight is not None:
        y = y * weight.double().reshape(shape)
    if bias is not None:
        y = y + bias.double().reshape(shape)
    if running_mean is not None:
        running_mean.mul_(1 - momentum).add_(momentum * mean.float())
        running_var.mul_(1 - momentum).add_(momentum * (var * count / max(count - 1, 1)).float())
    y = y.float()
    if out is not None:
        out.copy_(y)
        return out
    return y


def matmul_splitk(a, b, out=None):
    r = (a.double() @ b.double()).float()
    if out is not None:
        out.copy_(r)
        return out
    return r


def cross_entropy_partial(logits, targets, ignore_index=-100):
    x = logits.double()
    keep = targets != ignore_index
    lse = torch.logsumexp(x, dim=1)
    picked = x.gather(1, targets.clamp(0, x.shape[1] - 1).unsqueeze(1)).squeeze(1)
    loss = torch.where(keep, lse - picked, torch.zeros_like(lse))
    return torch.stack([loss.sum(), keep.double().sum()])


def cross_entropy_finalize(total, out=None):
    y = (total[0] / total[1]).float()
    if out is not None:
        out.copy_(y)
        return out
    return y
