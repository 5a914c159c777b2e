"""Expert-parallel MoE layer over the GPUs of one node, one process per GPU.

Rank r of a W-rank group owns e_rank global experts (e_rank defaults to 256 / W, so W ranks hold
the full 256-expert layer): by default the contiguous range [r * e_rank, (r + 1) * e_rank), or
the r-th list of an explicit placement (``balanced_placement`` spreads experts by expected load).
Each rank brings its own tokens.
``ExpertParallel.forward`` returns, for those tokens, the layer output over every owned expert
of every rank. The data path is the library's own kernels: token rows go to the owners and
partial results come back as peer stores over NVLink (CUDA IPC mappings); the ranks
synchronise through epoch flags in device memory. torch.distributed (NCCL or gloo) is used
only at set-up, to all-gather the IPC handles, and for the host barriers around set-up and
teardown.

Per rank the result equals, bit for bit, the fp32 sum over owner ranks d in ascending order of
``moe_forward(all tokens, experts of d, local_expert_offset = d * e_rank, fp32_out=True)``
(the fp32 per-token sum before moe_forward's final rounding), restricted to the rank's tokens
and rounded once to bf16. There is no counterpart in the reference, which runs one GPU with 32
local experts (kernels/moe.cu:744-900); each owner's share is exactly that computation.
"""
from __future__ import annotations

import ctypes

import torch

from . import _native
from .layer import (E_GLOBAL, G1_BLOCKS, H, H_BLOCKS, I_BLOCKS, W13_PACKED_SHAPE,
                    W2_PACKED_SHAPE, _cached_pack, _check, pack_w13, pack_w2)

MAX_RANKS = 8
EP_EVENTS = ["route", "dispatch", "arrive_barrier", "gather", "gemm1_swiglu", "gemm2_weighted",
             "combine_send", "done_barrier", "final_combine"]


def token_range(T_global: int, world: int, rank: int) -> tuple[int, int]:
    """Rows [lo, hi) of a T_global-token batch held by `rank` (even split, the first
    T_global % world ranks hold one more)."""
    _check(world >= 1 and 0 <= rank < world and T_global >= 0, "bad token partition")
    base, extra = divmod(T_global, world)
    lo = rank * base + min(rank, extra)
    return lo, lo + base + (1 if rank < extra else 0)


def expert_range(rank: int, e_rank: int) -> tuple[int, int]:
    """Global experts [lo, hi) owned by `rank`."""
    return rank * e_rank, (rank + 1) * e_rank


def owner_of(expert: int, world: int, e_rank: int) -> int:
    """Rank owning global expert `expert`, or -1 if no rank holds it."""
    return expert // e_rank if 0 <= expert < world * e_rank else -1


def exchange_handles(handle: bytes, group=None) -> list[bytes]:
    """All ranks' fixed-size handle blobs in rank order (one all_gather). With NCCL the blob
    travels as a uint8 tensor on the current CUDA device, with gloo on the CPU."""
    import torch.distributed as dist
    world = dist.get_world_size(group)
    backend = dist.get_backend(group)
    dev = torch.device("cuda", torch.cuda.current_device()) if backend == "nccl" else torch.device("cpu")
    mine = torch.tensor(list(handle), dtype=torch.uint8, device=dev)
    parts = [torch.empty_like(mine) for _ in range(world)]
    dist.all_gather(parts, mine, group=group)
    return [bytes(p.cpu().tolist()) for p in parts]


def balanced_placement(loads, world: int, e_rank: int, experts=None) -> list[list[int]]:
    """Assign `experts` (default 0 .. world * e_rank - 1) to `world` ranks, e_rank each, so the
    ranks' summed expected loads (`loads[g]`, e.g. route counts of a calibration batch) are
    close: largest load first, each to the least-loaded rank with room (ties to the lower rank).
    Each rank's list is returned in ascending expert order."""
    experts = list(range(world * e_rank)) if experts is None else [int(g) for g in experts]
    _check(len(experts) == world * e_rank and len(set(experts)) == len(experts), "need world * e_rank distinct experts")
    order = sorted(experts, key=lambda g: (-float(loads[g]), g))
    bins = [[] for _ in range(world)]
    total = [0.0] * world
    for g in order:
        d = min((r for r in range(world) if len(bins[r]) < e_rank), key=lambda r: (total[r], r))
        bins[d].append(g)
        total[d] += float(loads[g])
    return [sorted(b) for b in bins]


def agree_shapes(t_rank_max: int, e_rank: int, group=None, device=None) -> list[tuple[int, int]]:
    """(t_rank_max, e_rank) of every rank, in rank order (one all_gather)."""
    import torch.distributed as dist
    backend = dist.get_backend(group)
    dev = (device if device is not None else torch.device("cuda", torch.cuda.current_device())) \
        if backend == "nccl" else torch.device("cpu")
    mine = torch.tensor([t_rank_max, e_rank], dtype=torch.int64, device=dev)
    parts = [torch.empty_like(mine) for _ in range(dist.get_world_size(group))]
    dist.all_gather(parts, mine, group=group)
    return [(int(p[0]), int(p[1])) for p in parts]


class ExpertParallel:
    """One rank's expert-parallel context (symmetric buffer, peer mappings, workspace).

    ``t_rank_max``: most tokens any call on this rank passes (ranks may differ; every rank's
    buffers are sized for the largest value over the group, since the layout of the peer
    buffers must be identical); ``e_rank``: experts per rank (default 256 // world, the same on
    every rank). Without an initialised process group it runs as a single rank. Collective:
    every rank of the group constructs it; use as a context manager or call ``close()`` on
    every rank.
    """

    def __init__(self, t_rank_max: int, e_rank: int | None = None, group=None,
                 device: torch.device | int | None = None, placement=None):
        import torch.distributed as dist
        self.group = group
        self.distributed = dist.is_available() and dist.is_initialized()
        self.rank = dist.get_rank(group) if self.distributed else 0
        self.world = dist.get_world_size(group) if self.distributed else 1
        _check(1 <= self.world <= MAX_RANKS, "expert parallelism supports 1..8 ranks")
        self.e_rank = int(e_rank) if e_rank is not None else E_GLOBAL // self.world
        self.device = torch.device("cuda", torch.cuda.current_device() if device is None else
                                   (device if isinstance(device, int) else device.index))
        # All ranks agree on the buffer geometry before any of them allocates: the largest
        # t_rank_max of the group, and one e_rank (every rank sees the same gathered values, so
        # a mismatch raises on all of them and no rank is left waiting in a collective).
        shapes = agree_shapes(int(t_rank_max), self.e_rank, group, self.device) if self.world > 1 \
            else [(int(t_rank_max), self.e_rank)]
        _check(len({e for _, e in shapes}) == 1, f"e_rank differs between ranks: {[e for _, e in shapes]}")
        self.t_rank_max = max(1, max(t for t, _ in shapes))
        if placement is None:
            placement = [list(range(r * self.e_rank, (r + 1) * self.e_rank)) for r in range(self.world)]
        _check(len(placement) == self.world and all(len(p) == self.e_rank for p in placement),
               "placement must hold world lists of e_rank experts")
        self.placement = [[int(g) for g in p] for p in placement]
        flat = [g for p in self.placement for g in p]
        if self.world > 1:       # every rank must use the same table
            digest = int.from_bytes(__import__("hashlib").sha256(bytes(str(flat), "ascii")).digest()[:7], "little")
            seen = agree_shapes(digest, self.e_rank, group, self.device)
            _check(len({d for d, _ in seen}) == 1, "placement differs between ranks")
        self.lib = _native.cuda_lib()
        self._ctx = ctypes.c_void_p()
        handle = ctypes.create_string_buffer(_native.EP_HANDLE_BYTES)
        with torch.cuda.device(self.device):
            table = (ctypes.c_int * len(flat))(*flat)
            rc = self.lib.moe_ep_create(self.rank, self.world, self.t_rank_max, self.e_rank, table,
                                        ctypes.byref(self._ctx), handle)
            msg = self.lib.moe_last_error().decode(errors="replace") if rc else ""
            # A failure on any rank fails every rank here, before anyone waits on a peer.
            self._all_ok(rc == 0, f"moe_ep_create: {msg}")
            try:
                handles = (exchange_handles(handle.raw, group) if self.world > 1 else [handle.raw])
                rc = self.lib.moe_ep_connect(self._ctx, b"".join(handles))
                msg = self.lib.moe_last_error().decode(errors="replace") if rc else ""
                self._all_ok(rc == 0, f"moe_ep_connect: {msg}")
            except BaseException:
                self.lib.moe_ep_destroy(self._ctx)
                self._ctx = None
                raise
            nbytes = int(self.lib.moe_ep_workspace_bytes(self.world, self.t_rank_max, self.e_rank))
            self.workspace = torch.empty((nbytes,), dtype=torch.uint8, device=self.device)
        if self.world > 1:
            dist.barrier(group)       # every rank mapped every buffer before any forward

    def _all_ok(self, ok: bool, msg: str) -> None:
        """Raise on every rank unless every rank reports ok (one all_gather)."""
        flags = [ok]
        if self.world > 1:
            flags = [bool(t) for t, _ in agree_shapes(int(ok), self.e_rank, self.group, self.device)]
        if not all(flags):
            bad = [r for r, f in enumerate(flags) if not f]
            raise _native.MoEError(msg if not ok else f"expert-parallel set-up failed on rank(s) {bad}")

    @property
    def experts(self) -> list[int]:
        """Global experts of this rank, in the order of its weight arguments."""
        return list(self.placement[self.rank])

    def forward(self, hidden, hidden_scale, W13_packed, W13_scale, W2_packed, W2_scale, logits, bias,
                rsf: float, out: torch.Tensor | None = None, events=None, check: bool = False) -> torch.Tensor:
        """Layer output bf16 [T, 7168] for this rank's T tokens (moe_forward's argument order
        without local_expert_offset: this rank's experts are implied by its rank).

        The forward is asynchronous and never waits on the host. A peer that does not reach a
        flag barrier within the device wait limit makes the barrier give up: the device status
        word then holds ST_EP_TIMEOUT (16) and this forward's output rows are NaN. With
        ``check=True`` the call synchronises, reads (and clears) the status word and raises
        MoEError when any bit is set."""
        _check(self._ctx is not None, "expert-parallel context is closed")
        _check(hidden.dim() == 2 and int(hidden.size(1)) == H, "hidden must be [T, 7168]")
        T = int(hidden.size(0))
        _check(T <= self.t_rank_max, f"T must be at most t_rank_max ({self.t_rank_max})")
        _check(hidden.element_size() == 1, "hidden must be an FP8 tensor")
        _check(hidden_scale.dtype == torch.float32 and tuple(hidden_scale.shape) == (H_BLOCKS, T),
               "hidden_scale must be float32 [56, T]")
        _check(logits.dtype == torch.float32 and tuple(logits.shape) == (T, E_GLOBAL),
               "logits must be float32 [T, 256]")
        _check(bias.dtype == torch.float32 and bias.numel() == E_GLOBAL, "bias must be float32 [256]")
        E = self.e_rank
        _check(W13_packed.dtype == torch.uint8 and tuple(W13_packed.shape) == (E, *W13_PACKED_SHAPE),
               f"W13_packed must be [{E}, 16, 56, 256, 128] from pack_w13")
        _check(W2_packed.dtype == torch.uint8 and tuple(W2_packed.shape) == (E, *W2_PACKED_SHAPE),
               f"W2_packed must be [{E}, 28, 16, 256, 128] from pack_w2")
        _check(W13_scale.dtype == torch.float32 and tuple(W13_scale.shape) == (E, G1_BLOCKS, H_BLOCKS),
               f"W13_scale must be float32 [{E}, 32, 56]")
        _check(W2_scale.dtype == torch.float32 and tuple(W2_scale.shape) == (E, H_BLOCKS, I_BLOCKS),
               f"W2_scale must be float32 [{E}, 56, 16]")
        for t, n in ((hidden, "hidden"), (hidden_scale, "hidden_scale"), (W13_packed, "W13_packed"),
                     (W13_scale, "W13_scale"), (W2_packed, "W2_packed"), (W2_scale, "W2_scale"),
                     (logits, "logits"), (bias, "bias")):
            _check(t.is_cuda and t.device == self.device, f"{n} must be on {self.device}")
            _check(t.is_contiguous(), f"{n} must be contiguous")
        if out is None:
            out = torch.empty((T, H), dtype=torch.bfloat16, device=self.device)
        _check(out.dtype == torch.bfloat16 and tuple(out.shape) == (T, H) and out.is_contiguous(),
               "out must be a contiguous bf16 [T, 7168] tensor")
        args = (self._ctx, hidden.data_ptr(), hidden_scale.data_ptr(), W13_packed.data_ptr(),
                W13_scale.data_ptr(), W2_packed.data_ptr(), W2_scale.data_ptr(), logits.data_ptr(),
                bias.data_ptr(), float(rsf), T, out.data_ptr(), self.workspace.data_ptr(),
                self.workspace.numel(), torch.cuda.current_stream(self.device).cuda_stream)
        with torch.cuda.device(self.device):
            if events is None:
                _native.check(self.lib.moe_ep_forward(*args))
            else:
                _check(len(events) == len(EP_EVENTS) + 1, "events must hold 10 CUDA events")
                arr = (ctypes.c_void_p * len(events))(*[e.cuda_event for e in events])
                _native.check(self.lib.moe_ep_forward_profiled(*args, arr))
            if check:
                status = _native.device_status(reset=True)
                if status:
                    raise _native.MoEError(f"expert-parallel forward reported device status {status} "
                                           "(16 = a peer did not reach a barrier in time)")
        return out

    @torch.no_grad()
    def run(self, routing_logits, routing_bias, hidden_states, hidden_states_scale, gemm1_weights,
            gemm1_weights_scale, gemm2_weights, gemm2_weights_scale,
            routed_scaling_factor: float) -> torch.Tensor:
        """``reference.run``'s keyword surface for this rank: its tokens and its own experts'
        weights (packed once through the packed-weight cache)."""
        _check(int(gemm1_weights.shape[0]) == self.e_rank, f"gemm1_weights must hold {self.e_rank} experts")
        w13p = _cached_pack("w13", gemm1_weights, pack_w13)
        w2p = _cached_pack("w2", gemm2_weights, pack_w2)
        return self.forward(
            hidden_states.contiguous(), hidden_states_scale.to(torch.float32).contiguous(), w13p,
            gemm1_weights_scale.to(torch.float32).contiguous(), w2p,
            gemm2_weights_scale.to(torch.float32).contiguous(),
            routing_logits.to(torch.float32).contiguous(),
            routing_bias.to(torch.float32).reshape(-1).contiguous(), float(routed_scaling_factor))

    def close(self) -> None:
        """Collective: every rank's work is finished before any buffer is unmapped."""
        if self._ctx is None:
            return
        torch.cuda.synchronize(self.device)
        if self.world > 1:
            import torch.distributed as dist
            dist.barrier(self.group)
        rc = self.lib.moe_ep_destroy(self._ctx)
        self._ctx = None
        self.workspace = None
        _native.check(rc)

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()
