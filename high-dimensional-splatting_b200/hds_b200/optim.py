"""The optimizer step of the reference's training loop (gaussian_splatting/main.py:194,
torch.optim.Adam(fused=True, eps=1e-15) over one parameter group per tensor) as one kernel.

FlatAdam moves the storage of every parameter tensor into one flat fp32 buffer (the tensors stay
the same leaf objects, now views of it), keeps both Adam moments as flat buffers of the same
length, and reads the gradients from the flat GradBucket the backward passes accumulate into.  A
step is then a single memory-bound pass over all of them (hds_adam_step): 28 bytes per element.
"""
from __future__ import annotations

import ctypes

import numpy as np
import torch

from .native import check, lib, ptr, stream_of
from .parallel import GradBucket

# One learning rate per group, as the reference's GaussianModel.get_optimizer_params
# (utils/gaussian.py:123-139) and TrainingParams (config.py) set them; the means' rate is scaled by the
# scene extent.  The reference trains no feature table; it steps here at the SH DC rate.
REFERENCE_LRS = {"means": 0.00016, "log_scales": 0.005, "quats": 0.001, "opacity_logits": 0.025,
                 "sh_dc": 0.0025, "sh_rest": 0.0025 / 20, "features": 0.0025}
MAX_SEGMENTS = 16


def adam_step(params: torch.Tensor, exp_avg: torch.Tensor, exp_avg_sq: torch.Tensor, grads: torch.Tensor,
              segment_ends, segment_lrs, step: int, betas=(0.9, 0.999), eps: float = 1e-15) -> None:
    """One Adam step over flat [n] fp32 CUDA buffers (updated in place); segment s of the buffers,
    [segment_ends[s-1], segment_ends[s]), steps with learning rate segment_lrs[s]."""
    for t, name in ((params, "params"), (exp_avg, "exp_avg"), (exp_avg_sq, "exp_avg_sq"), (grads, "grads")):
        if not (t.is_cuda and t.dtype == torch.float32 and t.is_contiguous() and t.dim() == 1):
            raise RuntimeError(f"{name} must be a contiguous 1-D float32 CUDA tensor")
        if t.numel() != params.numel():
            raise RuntimeError(f"{name} has {t.numel()} elements, params {params.numel()}")
    k = len(segment_ends)
    if k != len(segment_lrs):
        raise RuntimeError("one learning rate per segment")
    ends = (ctypes.c_int64 * k)(*[int(e) for e in segment_ends])
    lrs = (ctypes.c_float * k)(*[float(x) for x in segment_lrs])
    b1, b2 = betas
    check(lib.hds_adam_step(params.numel(), ptr(params), ptr(exp_avg), ptr(exp_avg_sq), ptr(grads), k, ends, lrs,
                            float(step), float(b1), float(b2), float(np.float32(1.0 - b1)),
                            float(np.float32(1.0 - b2)), float(eps), stream_of(params.device)))


class FlatAdam:
    """Adam over a list of leaf parameters, with one learning rate per parameter (group).

    On construction every parameter's data moves into one flat buffer (`self.flat`, in list order)
    and, unless a bucket over the same parameters is given, a GradBucket is made for their gradients.
    step() runs one kernel over all parameters; lrs can change between steps (set_lr).

    head, tail: zero elements placed before and after the parameters in the flat buffer and in the
    gradient bucket (not stepped, no moments): room for rows that are rendered, and differentiated,
    beside the parameters' own (the tile-row split's fetched feature rows, which sort before and after
    the owned block)."""

    def __init__(self, params: list[torch.Tensor], lrs: list[float], betas=(0.9, 0.999), eps: float = 1e-15,
                 bucket: GradBucket | None = None, tail: int = 0, head: int = 0):
        if not params or len(params) != len(lrs):
            raise ValueError("one learning rate per parameter")
        if len(params) > MAX_SEGMENTS:
            raise ValueError(f"at most {MAX_SEGMENTS} parameters")
        dev = params[0].device
        for p in params:
            if not (p.is_leaf and p.dtype == torch.float32 and p.device == dev):
                raise ValueError("parameters must be float32 leaves on one device")
        self.params = params
        self.lrs = [float(x) for x in lrs]
        self.betas = betas
        self.eps = eps
        if (head or tail) and bucket is not None:
            raise ValueError("a head or tail needs the optimizer's own bucket")
        with torch.no_grad():
            self.flat = torch.cat(([torch.zeros(head, dtype=torch.float32, device=dev)] if head else []) +
                                  [p.detach().reshape(-1) for p in params] +
                                  ([torch.zeros(tail, dtype=torch.float32, device=dev)] if tail else [])).contiguous()
        ends, off = [], 0
        for p in params:
            n = p.numel()
            p.data = self.flat[head + off:head + off + n].view_as(p)
            off += n
            ends.append(off)
        self.segment_ends = ends
        self.n = off
        self.head = head
        self.exp_avg = torch.zeros(off, dtype=torch.float32, device=dev)
        self.exp_avg_sq = torch.zeros_like(self.exp_avg)
        if bucket is None:
            bucket = GradBucket(params, capacity=head + off + tail, offset=head)
        elif bucket.flat.numel() != off or any(a is not b for a, b in zip(bucket.params, params)):
            raise ValueError("the bucket must cover the same parameters in the same order")
        self.bucket = bucket
        self.step_count = 0

    @classmethod
    def from_buffers(cls, shapes: list[tuple], flat: torch.Tensor, exp_avg: torch.Tensor, exp_avg_sq: torch.Tensor,
                     lrs: list[float], step_count: int = 0, betas=(0.9, 0.999), eps: float = 1e-15) -> "FlatAdam":
        """A FlatAdam over existing flat buffers (e.g. written by hds_densify_apply): new leaf tensors of
        the given shapes as views of `flat`, with their own gradient bucket, and the given moments."""
        self = cls.__new__(cls)
        self.flat, self.exp_avg, self.exp_avg_sq = flat, exp_avg, exp_avg_sq
        self.n, self.head = flat.numel(), 0
        self.lrs, self.betas, self.eps, self.step_count = [float(x) for x in lrs], betas, eps, step_count
        params, ends, off = [], [], 0
        for shape in shapes:
            n = 1
            for d in shape:
                n *= d
            params.append(flat[off:off + n].view(shape).detach().requires_grad_(True))
            off += n
            ends.append(off)
        if off != flat.numel():
            raise ValueError("the shapes do not cover the flat buffer")
        self.params, self.segment_ends = params, ends
        self.bucket = GradBucket(params)
        return self

    def set_lr(self, index: int, lr: float) -> None:
        self.lrs[index] = float(lr)

    def zero_grad(self) -> None:
        self.bucket.zero()

    @torch.no_grad()
    def step(self) -> None:
        self.bucket.ready()
        self.step_count += 1
        h, n = self.head, self.n
        adam_step(self.flat[h:h + n], self.exp_avg, self.exp_avg_sq, self.bucket.flat[h:h + n], self.segment_ends,
                  self.lrs, self.step_count, self.betas, self.eps)


def shard_segments(segment_ends, lo: int, length: int) -> list[int]:
    """The segment ends of a flat buffer's slice [lo, lo + length), relative to the slice; the last
    segment is extended to the slice's end (zero padding past the parameters steps as a no-op)."""
    ends = [min(max(int(e) - lo, 0), length) for e in segment_ends]
    ends[-1] = length
    return ends


class ShardedFlatAdam:
    """FlatAdam for data parallelism over a process group: each rank steps 1/world of the flat
    parameter buffer.

    step() reduce-scatters the gradient bucket (every rank receives the sum over ranks of its shard),
    runs the Adam kernel over its shard with its own shard of both moments, and all-gathers the
    stepped shards back into every rank's full parameter buffer.  On the wire this is an all-reduce
    (a reduce-scatter plus an all-gather); the optimizer's memory traffic and the moments' storage
    per rank are 1/world of FlatAdam's.  Element for element the update is FlatAdam's applied to the
    all-reduced gradients."""

    ALIGN = 64  # elements: shards start on 256-byte boundaries

    def __init__(self, params: list[torch.Tensor], lrs: list[float], group=None, betas=(0.9, 0.999),
                 eps: float = 1e-15):
        import torch.distributed as dist

        if not params or len(params) != len(lrs):
            raise ValueError("one learning rate per parameter")
        if len(params) > MAX_SEGMENTS:
            raise ValueError(f"at most {MAX_SEGMENTS} parameters")
        dev = params[0].device
        for p in params:
            if not (p.is_leaf and p.dtype == torch.float32 and p.device == dev):
                raise ValueError("parameters must be float32 leaves on one device")
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.params, self.lrs, self.betas, self.eps = params, [float(x) for x in lrs], betas, eps
        n = sum(p.numel() for p in params)
        per = -(-n // self.world)
        self.shard = -(-per // self.ALIGN) * self.ALIGN
        padded = self.shard * self.world
        with torch.no_grad():
            self.flat = torch.zeros(padded, dtype=torch.float32, device=dev)
            ends, off = [], 0
            for p in params:
                k = p.numel()
                self.flat[off:off + k].copy_(p.detach().reshape(-1))
                p.data = self.flat[off:off + k].view_as(p)
                off += k
                ends.append(off)
        self.segment_ends = ends
        self.bucket = GradBucket(params, capacity=padded)
        self.lo = self.rank * self.shard
        self.local_ends = shard_segments(ends, self.lo, self.shard)
        self.exp_avg = torch.zeros(self.shard, dtype=torch.float32, device=dev)
        self.exp_avg_sq = torch.zeros_like(self.exp_avg)
        self.grad_shard = torch.empty_like(self.exp_avg)
        self.step_count = 0

    def set_lr(self, index: int, lr: float) -> None:
        self.lrs[index] = float(lr)

    def zero_grad(self) -> None:
        self.bucket.zero()

    @torch.no_grad()
    def step(self) -> None:
        import torch.distributed as dist

        self.bucket.ready()
        dist.reduce_scatter_tensor(self.grad_shard, self.bucket.flat, group=self.group)
        self.step_count += 1
        mine = self.flat[self.lo:self.lo + self.shard]
        adam_step(mine, self.exp_avg, self.exp_avg_sq, self.grad_shard, self.local_ends, self.lrs, self.step_count,
                  self.betas, self.eps)
        dist.all_gather_into_tensor(self.flat, mine, group=self.group)
