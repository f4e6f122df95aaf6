"""Multi-GPU plumbing: one process per GPU, torch.distributed (NCCL over
NVLink / NVSwitch) for the exchanges, the library's kernels for the compute.

The reference runs on one device only (its fusion windows bind to the first
SM120 device that runs a graph); tensor and expert parallelism are new here.

* Tensor-parallel dense FFN (config 2), sharded over the FFN width F = n_ff:
  rank r owns gate/up rows [r*F/P, (r+1)*F/P) and, of every down row, the
  NVFP4 blocks of columns [r*F/P, (r+1)*F/P).  Each rank computes its GLU
  columns and the down product over its K range locally; the P partial
  outputs are summed in rank order (one exchange per layer).  F/P is a
  multiple of 64, so the GLU's q8_1 blocks are the ones one GPU would make.
  `TpFfn` runs the step through the library (the partial outputs travel by
  NVLink peer stores from the down matvec's epilogue); `tp_ffn` is the same
  sharding over torch.distributed collectives with pluggable kernels.
* Expert-parallel MoE (config 3): rank r owns experts [r*E/P, (r+1)*E/P) and
  its own tokens.  Routing is computed locally (replicated router weights);
  each routed slot's activation row goes to the expert's owner (all-to-all),
  the owner runs its experts on the rows it received, the outputs come back
  (all-to-all) and the token's owner combines them in slot order -- the same
  arithmetic, in the same order, as the single-GPU fused layer.

`Kernels` bundles the compute calls; `GpuKernels` (the default) goes through
the C-ABI.  The exchange logic takes any object with the same methods, which is
how the CPU tests drive it over gloo.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

import ctypes as C

import numpy as np

from . import (_ptr, _stream, call, gemv_swiglu, lib, moe_combine, moe_experts, moe_route, mul_mat, quantize_q8_1)


class GpuKernels:
    """Compute through libfrb200 (CUDA tensors)."""

    def gate_up(self, x, wg, wu, n_rows, K):
        q8 = quantize_q8_1(x)
        return gemv_swiglu(wg, wu, q8, n_rows, K, x.shape[0])

    def down(self, glu, wd, n_rows, K):
        return mul_mat(wd, glu, n_rows, K)

    def route(self, x, w_r, n_used, clamp):
        _, ids, wts, _, _, _ = moe_route(x, w_r, n_used, clamp)
        return ids, wts

    def experts(self, x, eid, wg, wu, wd, n_embd, n_ff, E):
        return moe_experts(x, eid, wg, wu, wd, n_embd, n_ff, E)

    def combine(self, part, wts, n_embd, resid=None):
        return moe_combine(part, wts, n_embd, resid=resid)


def shard_range(n: int, rank: int, world: int):
    """Contiguous shard [lo, hi) of n items for `rank`; n % world == 0 required."""
    if n % world:
        raise ValueError(f"{n} rows do not split over {world} ranks")
    per = n // world
    return rank * per, (rank + 1) * per


def down_shard(wd, n_embd: int, n_ff: int, rank: int, world: int):
    """The K-shard of the down matrix [n_embd, n_ff/64 blocks of 36 bytes]
    that rank `rank` holds: blocks [rank*nb, (rank+1)*nb), nb = n_ff/64/world,
    as a contiguous [n_embd, nb*36] byte matrix (numpy or torch)."""
    if n_ff % (64 * world):
        raise ValueError(f"n_ff={n_ff} does not split into whole NVFP4 blocks over {world} ranks")
    nb = n_ff // 64 // world
    v = wd.reshape(n_embd, n_ff // 64, 36)[:, rank * nb:(rank + 1) * nb, :]
    if isinstance(v, torch.Tensor):
        return v.contiguous().reshape(n_embd, nb * 36)
    return np.ascontiguousarray(v).reshape(n_embd, nb * 36)


def _sum_over_ranks(part: torch.Tensor, world: int, group=None) -> torch.Tensor:
    """Sum of every rank's `part`, added in rank order (the same result on
    every rank)."""
    buf = torch.empty((world,) + tuple(part.shape), dtype=part.dtype, device=part.device)
    dist.all_gather_into_tensor(buf.view(world * part.shape[0], *part.shape[1:]), part.contiguous(), group=group)
    out = buf[0].clone()
    for r in range(1, world):
        out += buf[r]
    return out


def tp_ffn(x, wg_shard, wu_shard, wd_kshard, n_embd, n_ff, resid=None, group=None, kernels=None):
    """FFN sharded over n_ff; x [T, n_embd] replicated, wd_kshard from
    `down_shard`.  Returns the full output [T, n_embd] on every rank."""
    k = kernels or GpuKernels()
    world = dist.get_world_size(group)
    F_p = n_ff // world
    glu_shard = k.gate_up(x, wg_shard, wu_shard, F_p, n_embd)
    part = k.down(glu_shard, wd_kshard, n_embd, F_p)
    y = _sum_over_ranks(part, world, group)
    return y if resid is None else y + resid


class _PeerBuffer:
    """One device buffer per rank, mapped into every other rank's process by
    CUDA IPC (no multicast object); `peer_ptrs` is the device array of the
    ranks' base addresses the library's multi-GPU entries take."""

    def __init__(self, nbytes, group=None):
        import torch
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.nbytes = int(nbytes)
        if self.nbytes <= 0:
            raise ValueError("bad exchange buffer size")
        local = C.c_void_p()
        handle = (C.c_ubyte * 64)()
        call("fr_ipc_alloc", self.nbytes, C.byref(local), handle)
        self.local = local.value
        handles = [None] * self.world
        dist.all_gather_object(handles, bytes(handle), group=group)
        self.opened = []
        ptrs = []
        for r, h in enumerate(handles):
            if r == self.rank:
                ptrs.append(self.local)
                continue
            p = C.c_void_p()
            hb = (C.c_ubyte * 64).from_buffer_copy(h)
            call("fr_ipc_open", hb, C.byref(p))
            self.opened.append(p.value)
            ptrs.append(p.value)
        self.peer_ptrs = torch.tensor(ptrs, dtype=torch.int64, device=torch.cuda.current_device())
        dist.barrier(group=group)

    def close(self):
        """Release the mappings (all ranks, after their last step has finished)."""
        import torch
        if self.local is None:
            return
        torch.cuda.synchronize()
        dist.barrier(group=self.group)
        for p in self.opened:
            call("fr_ipc_close", C.c_void_p(p))
        self.opened = []
        dist.barrier(group=self.group)
        call("fr_ipc_free", C.c_void_p(self.local))
        self.local = None


class TpFfn(_PeerBuffer):
    """Tensor-parallel dense FFN with the reduction fused into the down
    matvec's epilogue: each rank's down matvec stores its partial output rows
    straight into its slot on every rank over NVLink (CUDA IPC peer mappings,
    no multicast object) and counts finished CTAs into per-rank flags; a
    bounded wait kernel sums the slots in rank order.  No NCCL call on the
    step; the step is one stream of kernels and is CUDA-graph capturable.

    `max_tokens` sizes the shared buffer; every call must use the same token
    count on all ranks (ranks advance in lock step)."""

    def __init__(self, max_tokens, n_embd, n_ff, group=None):
        world = dist.get_world_size(group)
        super().__init__(lib().fr_tp_buffer_bytes(max_tokens, n_embd, n_ff, world), group)
        self.n_embd, self.n_ff, self.max_tokens = n_embd, n_ff, max_tokens

    def __call__(self, x, wg_shard, wu_shard, wd_kshard, sg=None, su=None, sd=None, resid=None, out=None,
                 stream=None, tiled=False):
        """One step.  tiled: the shards are tile-major (frb200.tile_nvfp4 of
        the gate/up row shards and of the down K-shard)."""
        import torch
        T = x.shape[0]
        if T > self.max_tokens:
            raise ValueError(f"{T} tokens > buffer capacity {self.max_tokens}")
        if out is None:
            out = torch.empty((T, self.n_embd), dtype=torch.float32, device=x.device)
        call("fr_tp_ffn_tiled" if tiled else "fr_tp_ffn_nvfp4", _ptr(x), _ptr(wg_shard), _ptr(wu_shard),
             _ptr(wd_kshard), _ptr(sg), _ptr(su), _ptr(sd), _ptr(resid), _ptr(out), T, self.n_embd, self.n_ff,
             self.world, self.rank, _ptr(self.peer_ptrs), C.c_void_p(self.local), self.nbytes, _stream(stream))
        return out


class TpFfnRows(_PeerBuffer):
    """Tensor-parallel dense FFN row-sharded over the ranks (fr_tp_ffn_rows):
    gate/up rows and down rows sharded, the q8_1 GLU and the output
    all-gathered by NVLink peer stores with bounded waits; bit-identical to
    the single-GPU dp4a FFN.  Weights: `row_shards` of the full matrices."""

    def __init__(self, max_tokens, n_embd, n_ff, group=None):
        world = dist.get_world_size(group)
        super().__init__(lib().fr_tp_rows_buffer_bytes(max_tokens, n_embd, n_ff, world), group)
        self.n_embd, self.n_ff, self.max_tokens = n_embd, n_ff, max_tokens

    def __call__(self, x, wg_shard, wu_shard, wd_shard, sg=None, su=None, sd=None, resid=None, out=None,
                 stream=None):
        import torch
        T = x.shape[0]
        if T > self.max_tokens:
            raise ValueError(f"{T} tokens > buffer capacity {self.max_tokens}")
        if out is None:
            out = torch.empty((T, self.n_embd), dtype=torch.float32, device=x.device)
        call("fr_tp_ffn_rows", _ptr(x), _ptr(wg_shard), _ptr(wu_shard), _ptr(wd_shard), _ptr(sg), _ptr(su),
             _ptr(sd), _ptr(resid), _ptr(out), T, self.n_embd, self.n_ff, self.world, self.rank,
             _ptr(self.peer_ptrs), C.c_void_p(self.local), self.nbytes, _stream(stream))
        return out


def row_shards(wg, wu, wd, n_embd, n_ff, rank, world):
    """This rank's rows of the gate/up [n_ff, .] and down [n_embd, .] matrices."""
    f0, f1 = shard_range(n_ff, rank, world)
    e0, e1 = shard_range(n_embd, rank, world)
    return wg[f0:f1].contiguous(), wu[f0:f1].contiguous(), wd[e0:e1].contiguous()


class EpMoe(_PeerBuffer):
    """Expert-parallel MoE layer over NVLink peer stores (fr_ep_moe_nvfp4):
    this rank's E/P experts, its own tokens; routed rows go to the expert
    owners and outputs come back through fixed-capacity exchange buffers, with
    bounded waits and no host synchronisation (CUDA-graph capturable).  The
    result equals the single-GPU layer.  Every call uses the same T on all
    ranks, T <= max_tokens."""

    def __init__(self, max_tokens, n_embd, n_ff, E, n_used, group=None):
        world = dist.get_world_size(group)
        if E % world:
            raise ValueError(f"{E} experts do not split over {world} ranks")
        super().__init__(lib().fr_ep_buffer_bytes(max_tokens, n_embd, n_used, world), group)
        self.max_tokens, self.n_embd, self.n_ff, self.E, self.n_used = max_tokens, n_embd, n_ff, E, n_used

    def __call__(self, x, w_r, wg_local, wu_local, wd_local, sg=None, su=None, sd=None, resid=None, out=None,
                 clamp=6.103515625e-5, stream=None, tiled=False):
        """tiled: the local experts are tile-major (frb200.tile_experts), run
        on the FP4 tensor cores (fr_ep_moe_tiled)."""
        import torch
        T = x.shape[0]
        if T > self.max_tokens:
            raise ValueError(f"{T} tokens > buffer capacity {self.max_tokens}")
        if out is None:
            out = torch.empty((T, self.n_embd), dtype=torch.float32, device=x.device)
        call("fr_ep_moe_tiled" if tiled else "fr_ep_moe_nvfp4", _ptr(x), _ptr(w_r), _ptr(wg_local), _ptr(wu_local), _ptr(wd_local), _ptr(sg), _ptr(su),
             _ptr(sd), _ptr(resid), _ptr(out), T, self.max_tokens, self.n_embd, self.n_ff, self.E, self.n_used,
             clamp, self.world, self.rank, _ptr(self.peer_ptrs), C.c_void_p(self.local), self.nbytes,
             _stream(stream))
        return out


def _exchange(send: torch.Tensor, send_counts, recv_counts, group=None) -> torch.Tensor:
    """Variable-size all-to-all of rows (counts are per peer, in rows)."""
    world = len(send_counts)
    width = send.shape[1:] if send.dim() > 1 else ()
    out = torch.empty((int(sum(recv_counts)),) + tuple(width), dtype=send.dtype, device=send.device)
    if dist.get_backend(group) == "nccl":
        dist.all_to_all_single(out, send.contiguous(), output_split_sizes=list(recv_counts),
                               input_split_sizes=list(send_counts), group=group)
        return out
    # backends without all_to_all: every rank gathers the padded send buffers
    mx = max(1, max(int(c) for c in send_counts), max(int(c) for c in recv_counts))
    pad = torch.zeros((world, mx) + tuple(width), dtype=send.dtype, device=send.device)
    offs = [0]
    for c in send_counts:
        offs.append(offs[-1] + int(c))
    rank = dist.get_rank(group)
    gathered = torch.empty((world, world, mx) + tuple(width), dtype=send.dtype, device=send.device)
    for p in range(world):
        pad[p, :int(send_counts[p])] = send[offs[p]:offs[p + 1]]
    dist.all_gather_into_tensor(gathered.view(world * world, mx, *width), pad.view(world, mx, *width), group=group)
    pieces = [gathered[src, rank, :int(recv_counts[src])] for src in range(world)]
    out.copy_(torch.cat(pieces, 0) if pieces else out)
    return out


def ep_moe(x, w_r, wg_local, wu_local, wd_local, n_embd, n_ff, E, n_used, resid=None,
           clamp=6.103515625e-5, group=None, kernels=None):
    """Expert-parallel MoE layer for this rank's tokens x [T, n_embd].
    wg/wu/wd_local hold this rank's E/P experts.  Returns [T, n_embd]."""
    k = kernels or GpuKernels()
    world = dist.get_world_size(group)
    E_p = E // world
    T = x.shape[0]
    ids, wts = k.route(x, w_r, n_used, clamp)                    # [T, n_used] global expert ids
    flat = ids.reshape(-1).long()
    dest = torch.div(flat, E_p, rounding_mode="floor")
    # stable order of the slots by destination rank (slot order inside a rank)
    order = torch.argsort(dest * (T * n_used) + torch.arange(T * n_used, device=flat.device))
    send_counts = torch.bincount(dest, minlength=world)
    counts = torch.empty((world, world), dtype=torch.int64, device=flat.device)
    dist.all_gather_into_tensor(counts.view(-1), send_counts.to(torch.int64).contiguous(), group=group)
    rank = dist.get_rank(group)
    sc = [int(v) for v in counts[rank].tolist()]
    rc = [int(v) for v in counts[:, rank].tolist()]
    tok = torch.div(order, n_used, rounding_mode="floor")
    send_x = x[tok]                                               # [S, n_embd] in send order
    send_e = (flat[order] - dest[order] * E_p).to(torch.int32)
    recv_x = _exchange(send_x, sc, rc, group)
    recv_e = _exchange(send_e.view(-1, 1), sc, rc, group).view(-1)
    y_recv = k.experts(recv_x.contiguous(), recv_e.contiguous(), wg_local, wu_local, wd_local, n_embd, n_ff, E_p)
    back = _exchange(y_recv, rc, sc, group)                       # rows in our send order
    part = torch.empty((T * n_used, n_embd), dtype=back.dtype, device=back.device)
    part[order] = back
    return k.combine(part, wts, n_embd, resid=resid)
