"""Row-sharded NVFP4 quantization across the GPUs of one node.

An activation X (rows x cols, row-major bf16) is split by row blocks across
the ranks of a torch.distributed group (one process per GPU).  In the API's
column-major view each rank holds an m x n_r matrix (m = cols, n_r = its rows),
i.e. columns [n_offset, n_offset + n_r) of the full m x n_total problem.  One
step is
    local amax (nvfp4_amax_bf16)
    -> combination of that scalar across the ranks, the only exchange:
       exchange="nccl", an NCCL int32-MAX all-reduce over NVLink between the
       two kernels; exchange="peer", inside the cast kernel, which publishes
       and reads the ranks' amax over NVLink peer memory
    -> RHT GEMM + NVFP4 cast of the shard with the full problem's RNG
       coordinates (nvfp4_rht_gemm_ntt_w_sfc_sharded[_exchange]),
so the per-rank outputs concatenated along the column dimension equal the
single-GPU result bit for bit.  With fused=True one kernel computes the
shard's amax, exchanges it over peer memory and casts.  The reference has no
multi-GPU path; this follows the row-sharding its north-star configuration
asks for.
"""
from __future__ import annotations

import contextlib
from dataclasses import dataclass
from datetime import timedelta
from typing import Callable, Optional

import torch
import torch.distributed as dist


@dataclass(frozen=True)
class ShardPlan:
    m: int
    n_total: int
    world: int
    k_tile_size: int
    offsets: tuple
    sizes: tuple

    @property
    def chunk(self) -> int:
        """Column granularity that keeps TE's RNG coordinates shard-invariant."""
        return (min(self.n_total, self.k_tile_size) // 64) * 64


def plan_shards(m: int, n_total: int, world: int, k_tile_size: int = 2048) -> ShardPlan:
    """Split n_total columns into `world` contiguous shards whose offsets are
    multiples of the RNG chunk (min(n_total, k_tile_size) rounded down to 64).
    Shards may differ in size by one chunk; a rank may get zero columns."""
    if m % 128 or n_total % 64 or n_total <= 0 or world <= 0 or k_tile_size < 64:
        raise ValueError(f"bad problem: m={m} n_total={n_total} world={world} k_tile={k_tile_size}")
    chunk = (min(n_total, k_tile_size) // 64) * 64
    nchunks, rem = divmod(n_total, chunk)
    offsets, sizes, pos = [], [], 0
    for r in range(world):
        take = (nchunks // world + (1 if r < nchunks % world else 0)) * chunk
        if r == world - 1:
            take += rem
        offsets.append(pos)
        sizes.append(take)
        pos += take
    assert pos == n_total
    return ShardPlan(m, n_total, world, k_tile_size, tuple(offsets), tuple(sizes))


def combine_amax(local_amax: torch.Tensor, group=None) -> torch.Tensor:
    """Max-allreduce of the scalar amax, in place, as one int32 MAX collective
    on the float's bit pattern: amax is never negative, so the signed order of
    the bits is the order of the values, and every NaN pattern sorts above
    +Inf -- a NaN on any rank yields NaN on every rank (NaN-propagating, like
    the amax kernels) without comparing floats."""
    if dist.is_available() and dist.is_initialized() and dist.get_world_size(group) > 1:
        assert local_amax.dtype == torch.float32 and local_amax.is_contiguous()
        dist.all_reduce(local_amax.view(torch.int32), op=dist.ReduceOp.MAX, group=group)
    return local_amax


def stream_context(stream):
    """Make `stream` torch's current stream for the duration of a step.

    The amax kernel, the NCCL all-reduce and the cast must be ordered on ONE
    stream: torch.distributed enqueues the all-reduce on torch's current
    stream, so a step given another stream runs entirely inside this context.
    `stream` may be None (the current stream), a torch.cuda.Stream or a raw
    cudaStream_t handle."""
    if stream is None:
        return contextlib.nullcontext()
    if not isinstance(stream, torch.cuda.Stream):
        stream = torch.cuda.ExternalStream(int(stream))
    return torch.cuda.stream(stream)


class ShardedRhtQuantizer:
    """One rank's side of the row-sharded quantization step."""

    def __init__(self, m: int, n_total: int, *, group=None, k_tile_size: int = 2048,
                 stochastic_rounding: bool = True, use_fast_math: bool = False,
                 rng_state: Optional[torch.Tensor] = None, exchange: str = "nccl",
                 fused: bool = False):
        """exchange: "nccl" -- int32-MAX allreduce of the amax before the cast;
        "peer" -- the cast kernel itself publishes and combines the amax over
        NVLink peer memory (every rank needs a non-empty shard).
        fused: one kernel computes the shard's amax and casts (single GPU, or
        with exchange="peer")."""
        self.group = group
        world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.plan = plan_shards(m, n_total, world, k_tile_size)
        self.m, self.n_total = m, n_total
        self.n_offset = self.plan.offsets[self.rank]
        self.n = self.plan.sizes[self.rank]
        self.k_tile_size = k_tile_size
        self.sr, self.fm = stochastic_rounding, use_fast_math
        self.rng_state = rng_state
        self.peer = None
        self.fused = fused
        self.workspace = None
        world = self.plan.world
        if fused and world > 1 and exchange != "peer":
            raise ValueError("the fused kernel combines the ranks' amax over peer memory; "
                             "use exchange='peer'")
        if exchange == "peer" and world > 1:
            if min(self.plan.sizes) == 0:
                raise ValueError("the peer exchange needs a non-empty shard on every rank")
            from .ops import PeerExchange
            self.peer = PeerExchange(self.rank, world)
            handles = [None] * world
            dist.all_gather_object(handles, bytes(self.peer.handle.raw), group=group)
            self.peer.connect(handles)
            dist.barrier(group=group)
        elif exchange not in ("nccl", "peer"):
            raise ValueError(exchange)

    def outputs(self, device="cuda"):
        C = torch.empty((self.m, self.n // 2), dtype=torch.uint8, device=device)
        S = torch.empty((self.m, self.n // 16), dtype=torch.uint8, device=device)
        return C, S

    def __call__(self, A_shard: torch.Tensor, B: torch.Tensor, C: torch.Tensor, S: torch.Tensor,
                 amax: Optional[torch.Tensor] = None, stream=None,
                 local_amax_fn: Optional[Callable] = None, cast_fn: Optional[Callable] = None):
        """Quantize this rank's shard; returns the global amax tensor.
        local_amax_fn / cast_fn replace the CUDA kernels (tests run the host
        logic on CPU with them).  `stream` (None: torch's current stream) is
        made the current stream for the whole step, so that the all-reduce of
        the NCCL exchange is ordered between the amax kernel and the cast."""
        with stream_context(stream):
            return self._step(A_shard, B, C, S, amax, stream, local_amax_fn, cast_fn)

    def _step(self, A_shard, B, C, S, amax, stream, local_amax_fn, cast_fn):
        from . import ops
        if amax is None:
            amax = torch.empty(1, dtype=torch.float32, device=A_shard.device)
        if self.fused and cast_fn is None and local_amax_fn is None:
            if self.workspace is None:
                self.workspace = ops.fused_workspace(A_shard.device)
            if self.peer is not None:
                ops.quantize_rht_fused_sharded_exchange(
                    self.m, self.n, A_shard, B, C, S, amax, self.rng_state, self.n_offset,
                    self.n_total, self.peer, self.workspace, 0, stream, self.k_tile_size,
                    stochastic_rounding=self.sr, use_fast_math=self.fm)
            else:   # one rank: the shard is the whole matrix
                ops.quantize_rht_fused(self.m, self.n, A_shard, B, C, S, amax, self.rng_state,
                                       self.workspace, 0, stream, self.k_tile_size,
                                       stochastic_rounding=self.sr, use_fast_math=self.fm)
            return amax
        if local_amax_fn is None:
            ops.amax_bf16(A_shard, self.m * self.n, amax, stream)
        else:
            local_amax_fn(A_shard, amax)
        if self.peer is not None and cast_fn is None:
            # one kernel: publish this rank's amax, combine all ranks', cast
            ops.rht_gemm_ntt_w_sfc_sharded_exchange(
                self.m, self.n, A_shard, B, C, S, amax, amax, self.rng_state, self.n_offset,
                self.n_total, self.peer, 0, stream, self.k_tile_size,
                stochastic_rounding=self.sr, use_fast_math=self.fm)
            return amax
        combine_amax(amax, self.group)
        if cast_fn is None:
            if self.n > 0:
                ops.rht_gemm_ntt_w_sfc_sharded(self.m, self.n, A_shard, B, C, S, amax,
                                               self.rng_state, self.n_offset, self.n_total, 0,
                                               stream, self.k_tile_size,
                                               stochastic_rounding=self.sr,
                                               use_fast_math=self.fm)
        else:
            cast_fn(self, A_shard, B, C, S, amax)
        return amax


def init_distributed(backend: str = "nccl", timeout_s: float = 60.0):
    """One process per GPU; reads RANK / WORLD_SIZE / LOCAL_RANK / MASTER_* from
    the environment.  A rank that never joins makes the others' collectives
    fail after `timeout_s` instead of hanging."""
    import os
    local = int(os.environ.get("LOCAL_RANK", "0"))
    kw = {}
    if backend == "nccl":
        torch.cuda.set_device(local)
        kw["device_id"] = torch.device("cuda", local)
    dist.init_process_group(backend, timeout=timedelta(seconds=timeout_s), **kw)
    return dist.get_rank(), dist.get_world_size(), local
