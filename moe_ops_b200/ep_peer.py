"""Expert parallelism with dispatch and combine over NVLink peer memory.

The NCCL path in ``ep.py`` permutes locally, runs a row all-to-all, then regroups. Here
the GPUs write and read each other's buffers directly, and the routing bookkeeping never
reaches the host. Each rank's receive buffer is already the grouped GEMM's layout:
expert-major, then source-rank-major.

Per layer step (rank r of W, El = E / W local experts):

    forward   permute index pass (no copy) -> counts exchange (peer stores + B0)
              -> delta / offsets (tiny tensor ops) -> slot map
              -> dispatch: rows straight into the owners' receive buffers
              -> B2 -> gate/up + SwiGLU, down GEMMs into this rank's `down` buffer
              -> B3 -> combine: out[t] = sum_k w[t,k] * down row read from its owner
    backward  combine backward: w-scaled gradient rows pushed into the owners' `gdown`,
              routing-weight gradients from the owners' `down` rows
              -> B4 -> expert backward (fused dgrad + SwiGLU backward, wgrads)
              -> `dgrad` buffer -> B5 -> dispatch backward: pull and sum over k

The barriers Bi are device-side (``moe_ep_barrier``). Waits are bounded, and every buffer
reuse across ranks is ordered by one of them. For example, a rank's next dispatch into a
peer's receive buffer waits at B0 (the counts exchange of that step) until that peer's
previous backward has finished reading it.
Nothing in a step synchronises with the host or calls a collective library, and the
barriers keep their epochs on the device, so a whole training step (forward and backward)
can be captured in a CUDA graph and replayed.

Results equal the single-GPU layer on the concatenated tokens bit for bit. An expert sees
its rows in the same order (source rank, then stable slot order), and combine and its
backward use the unpermute kernels' rounding.

The transport is an interface, so that the data path can be tested with W ranks emulated
in one process on one GPU. The real one, ``NVLinkTransport``, maps the peers' buffers
through CUDA IPC (plain device memory, no multicast object).
"""
from __future__ import annotations

import ctypes

import torch
import torch.distributed as dist

from . import _lib

_KINDS = ("recv", "down", "gdown", "dgrad")
_MAX_COUNT_EXPERTS = 1024  # experts the counts exchange array holds


def _as_tensor(ptr: int, shape: tuple, dtype: torch.dtype, device: torch.device) -> torch.Tensor:
    """A torch view of device memory this library allocated (zero copy, not owned)."""
    code = {2: "<i2", 4: "<f4", 8: "<i8"}[torch.empty((), dtype=dtype).element_size()]

    class _Mem:
        __cuda_array_interface__ = {"shape": tuple(shape), "typestr": code, "data": (ptr, False),
                                    "version": 3, "strides": None}

    t = torch.as_tensor(_Mem(), device=device)
    return t if t.dtype == dtype else t.view(dtype)


class PeerTransport:
    """What the peer-memory EP step needs from the ranks around it."""

    rank: int
    world: int
    capacity: int          # rows of each row buffer
    buffers: dict          # kind -> this rank's [capacity, cols] tensor
    bases: dict            # kind -> device int64 [world]: every rank's buffer, mapped here

    def all_gather_counts(self, counts: torch.Tensor) -> torch.Tensor:
        """[E] int32 (device) -> [world, E] int32 (device), without a host sync."""
        raise NotImplementedError

    def barrier(self) -> None:
        raise NotImplementedError


class NVLinkTransport(PeerTransport):
    """One process per GPU. Row buffers and barrier flags live in this library's
    allocations. The peers map them through CUDA IPC once, so every later step only
    launches kernels."""

    def __init__(self, group, capacity: int, cols: int, dtype: torch.dtype, device,
                 timeout_s: float = 5.0):
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.capacity, self.cols, self.dtype = capacity, cols, dtype
        self.device = torch.device(device)
        self.timeout_ns = int(timeout_s * 1e9)
        lib = _lib.load()
        es = torch.empty((), dtype=dtype).element_size()
        # the row buffers, the counts exchange array [world, kMaxCountExperts] int32, the
        # barrier flags [world] int64
        sizes = ([capacity * cols * es] * len(_KINDS) + [4 * self.world * _MAX_COUNT_EXPERTS]
                 + [8 * self.world])
        self._own, handles = [], bytearray()
        with torch.cuda.device(self.device):
            for nbytes in sizes:
                ptr = ctypes.c_void_p()
                h = (ctypes.c_uint8 * 64)()
                _lib.check(lib.moe_ipc_malloc(nbytes, ctypes.byref(ptr), ctypes.addressof(h)),
                           "moe_ipc_malloc")
                self._own.append(ptr.value)
                handles += bytes(h)
            mine = torch.frombuffer(handles, dtype=torch.uint8).to(self.device)
            allh = torch.empty(self.world, mine.numel(), dtype=torch.uint8, device=self.device)
            dist.all_gather_into_tensor(allh, mine, group=group)
            allh = allh.cpu()
            self._opened = []
            table = [[0] * self.world for _ in sizes]
            for r in range(self.world):
                for i in range(len(sizes)):
                    if r == self.rank:
                        table[i][r] = self._own[i]
                        continue
                    h = (ctypes.c_uint8 * 64).from_buffer_copy(bytes(allh[r, 64 * i: 64 * (i + 1)].tolist()))
                    ptr = ctypes.c_void_p()
                    _lib.check(lib.moe_ipc_open(ctypes.addressof(h), ctypes.byref(ptr)), "moe_ipc_open")
                    self._opened.append(ptr.value)
                    table[i][r] = ptr.value
            self.buffers = {k: _as_tensor(self._own[i], (capacity, cols), dtype, self.device)
                            for i, k in enumerate(_KINDS)}
            self.bases = {k: torch.tensor(table[i], dtype=torch.int64, device=self.device)
                          for i, k in enumerate(_KINDS)}
            self._flags = _as_tensor(self._own[-1], (self.world,), torch.int64, self.device)
            self._flags.zero_()
            self._flag_table = torch.tensor(table[-1], dtype=torch.int64, device=self.device)
            self._epoch = torch.zeros(1, dtype=torch.int64, device=self.device)
            self._counts = _as_tensor(self._own[-2], (self.world * _MAX_COUNT_EXPERTS,),
                                      torch.int32, self.device)
            self._counts_table = torch.tensor(table[-2], dtype=torch.int64, device=self.device)
            self._status = torch.ones(1, dtype=torch.int32, device=self.device)
            # Health of the previous steps, copied to pinned host memory at the end of every
            # backward and read (without a sync) at the start of a later forward.
            self._health_host = torch.zeros(2, dtype=torch.int32).pin_memory()
            self._health_dev = torch.zeros(2, dtype=torch.int32, device=self.device)
            self._health_event = None
            torch.cuda.synchronize(self.device)
        self.step = 0                 # forwards run so far (a backward checks it)
        self.pending_backward = False
        dist.barrier(group=group)  # every rank's flags are zero before the first signal

    @property
    def status(self) -> torch.Tensor:
        """Device int32 [1]: 1 while every barrier so far completed, 0 after one gave up."""
        return self._status

    def all_gather_counts(self, counts):
        """Over peer memory, no collective library: this rank's counts go into row `rank` of
        every rank's exchange array, then a barrier.  The returned [world, E] view is valid
        until this rank's next call (every rank reads it before the step's later barriers)."""
        E = counts.numel()
        if E > _MAX_COUNT_EXPERTS:
            raise ValueError(f"at most {_MAX_COUNT_EXPERTS} experts")
        lib = _lib.load()
        counts = counts.to(torch.int32).contiguous()
        _lib.check(lib.moe_ep_put_counts(_lib.ptr(counts), E, _lib.ptr(self._counts_table),
                                         self.rank, self.world, _lib.stream_of(counts)),
                   "moe_ep_put_counts")
        _lib.count_launches(1)
        self.barrier()
        return self._counts[: self.world * E].view(self.world, E)

    def barrier(self):
        lib = _lib.load()
        st = lib.moe_ep_barrier(_lib.ptr(self._flag_table), self.rank, self.world,
                                _lib.ptr(self._epoch), self.timeout_ns, _lib.ptr(self._status),
                                _lib.stream_of(self._flag_table))
        _lib.check(st, "moe_ep_barrier")
        _lib.count_launches(1)

    def barrier_ok(self) -> bool:
        """False if any barrier so far gave up waiting (reads the status: syncs)."""
        return bool(self._status.item())

    def record_health(self) -> None:
        """Enqueues a copy of the barrier status and the library's device error word into
        pinned host memory (no sync); check_health() reads it once it has landed."""
        lib = _lib.load()
        stream = torch.cuda.current_stream(self.device)
        self._health_dev[:1].copy_(self._status)
        _lib.check(lib.moe_peek_device_error(_lib.ptr(self._health_dev[1:]), stream.cuda_stream),
                   "moe_peek_device_error")
        self._health_host.copy_(self._health_dev, non_blocking=True)
        self._health_event = torch.cuda.Event()
        self._health_event.record(stream)

    def check_health(self) -> None:
        """Raises if an earlier step's barrier gave up or a kernel raised a device error.
        Reads the last record_health() copy only if it has completed: never syncs."""
        ev = self._health_event
        if ev is None or not ev.query():
            return
        status, err = self._health_host.tolist()
        if status == 0 or err != 0:
            raise RuntimeError(
                f"EP peer transport (rank {self.rank}): an earlier step failed (barrier "
                f"status {status}, device error {err}); its results are not valid. Close the "
                "layer on every rank and rebuild it.")

    def close(self):
        """Collective: unmaps the peers' buffers, waits until every rank has done so, then
        frees this rank's own (an exporter must not free memory a peer still maps)."""
        if not self._own:
            return
        if self.pending_backward:
            raise RuntimeError("NVLinkTransport.close(): a forward's backward has not run yet; "
                               "it still needs these buffers")
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        lib = _lib.load()
        for p in self._opened:
            lib.moe_ipc_close(p)
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        for p in self._own:
            lib.moe_ipc_free(p)
        self._opened, self._own = [], []


def _layout(counts_all: torch.Tensor, offsets: torch.Tensor, rank: int, world: int):
    """From all ranks' per-expert counts [W, E]: delta[E] (this rank's rows of expert e
    move from offsets[e] to their row in the owner's receive buffer) and this rank's
    grouped-GEMM offsets [El + 1]."""
    W, E = counts_all.shape
    El = E // W
    cm = counts_all.view(W, W, El).to(torch.int64)            # [src, owner, local expert]
    tot = cm.sum(0)                                           # [owner, El]
    recv_base = torch.cumsum(tot, 1) - tot                    # [owner, El]
    src_off = torch.cumsum(cm, 0) - cm                        # [src, owner, El]
    delta = (recv_base + src_off[rank]).reshape(E) - offsets[:-1].to(torch.int64)
    off_local = torch.zeros(El + 1, dtype=torch.int32, device=counts_all.device)
    off_local[1:] = torch.cumsum(tot[rank], 0).to(torch.int32)
    return delta.to(torch.int32), off_local


class _PeerExperts(torch.autograd.Function):
    """The expert segment of an EP layer over peer memory:
    (x [T, d], routing weights [T, K], indices [T, K], local expert weights) -> out [T, d]."""

    @staticmethod
    def forward(ctx, x, weights, indices, w_gate, w_up, w_down, tr, num_experts):
        from .gate_up_ops import gmm_gate_up_fwd_raw
        from .grouped_gemm_ops import _gmm_call
        from .permute_ops import permute_countsort

        lib = _lib.load()
        T, d = x.shape
        K = indices.shape[1]
        E, W = num_experts, tr.world
        status = getattr(tr, "status", None)
        tr.step = getattr(tr, "step", 0) + 1
        ctx.step = tr.step
        tr.pending_backward = any(ctx.needs_input_grad)
        El = E // W
        x = x.contiguous()
        indices = indices.to(torch.int32).contiguous()
        _, rid, offsets = permute_countsort(x[:, :0], indices, 0, E)   # index pass only
        counts_all = tr.all_gather_counts(offsets[1:] - offsets[:-1])
        delta, off_local = _layout(counts_all, offsets, tr.rank, W)
        tr.last_local_rows = off_local[El:]  # rows this rank's experts compute on (device)
        ranks = torch.empty(T * K, dtype=torch.int32, device=x.device)
        rows = torch.empty_like(ranks)
        stream = _lib.stream_of(x)
        _lib.check(lib.moe_ep_slot_map(_lib.ptr(indices), _lib.ptr(rid), _lib.ptr(delta), T, K, E,
                                       El, W, tr.capacity, _lib.ptr(ranks), _lib.ptr(rows), stream),
                   "moe_ep_slot_map")
        dt = _lib.dtype_code(x.dtype)
        # No barrier before the dispatch: B0 (inside all_gather_counts) already waits for
        # every peer to have reached this step, so its previous backward has finished
        # reading the receive buffer this dispatch writes.
        _lib.check(lib.moe_ep_dispatch(_lib.ptr(x), dt, _lib.ptr(tr.bases["recv"]), _lib.ptr(ranks),
                                       _lib.ptr(rows), T, K, d, _lib.ptr(status), stream),
                   "moe_ep_dispatch")
        tr.barrier()                                               # B2
        recv, down = tr.buffers["recv"], tr.buffers["down"]
        gate, up, h = gmm_gate_up_fwd_raw(recv, w_gate, w_up, off_local, True)
        _gmm_call("moe_gmm_fwd", h, w_down, down, off_local, tr.capacity, w_down.shape[1],
                  w_down.shape[2], El, True)
        tr.barrier()                                               # B3
        out = torch.empty(T, d, device=x.device, dtype=x.dtype)
        w = weights.contiguous()
        _lib.check(lib.moe_ep_combine(_lib.ptr(tr.bases["down"]), dt, _lib.ptr(ranks), _lib.ptr(rows),
                                      _lib.ptr(w), _lib.dtype_code(w.dtype), T, K, d, _lib.ptr(out),
                                      _lib.ptr(status), stream), "moe_ep_combine")
        _lib.count_launches(3)
        ctx.save_for_backward(w, ranks, rows, off_local, gate, up, h, w_gate, w_up, w_down)
        ctx.tr, ctx.shape = tr, (T, K, d, El)
        return out

    @staticmethod
    def backward(ctx, grad_out):
        from .gate_up_ops import (dgrad_dual_into, dgrad_dual_ok, gmm_dgrad_swiglu_bwd_raw,
                                  run_on_side)
        from .grouped_gemm_ops import _gmm_call, gmm_bwd_B_raw, gmm_dgrad_raw

        w, ranks, rows, off_local, gate, up, h, w_gate, w_up, w_down = ctx.saved_tensors
        tr = ctx.tr
        if getattr(tr, "step", ctx.step) != ctx.step:
            # The transport's shared buffers (received rows, expert outputs) now hold a later
            # forward's rows: this backward would silently mix the two steps.
            raise RuntimeError(
                "EP peer transport: backward of forward step %d after step %d ran; the "
                "peer-memory layer needs each backward before the next forward" %
                (ctx.step, tr.step))
        status = getattr(tr, "status", None)
        T, K, d, El = ctx.shape
        lib = _lib.load()
        grad_out = grad_out.to(w_down.dtype).contiguous()
        stream = _lib.stream_of(grad_out)
        dt = _lib.dtype_code(grad_out.dtype)
        grad_w = torch.empty_like(w)
        _lib.check(lib.moe_ep_combine_bwd(_lib.ptr(grad_out), _lib.ptr(tr.bases["down"]),
                                          _lib.ptr(tr.bases["gdown"]), dt, _lib.ptr(ranks),
                                          _lib.ptr(rows), _lib.ptr(w), _lib.dtype_code(w.dtype), T, K,
                                          d, _lib.ptr(grad_w), _lib.ptr(status), stream),
                   "moe_ep_combine_bwd")
        tr.barrier()                                               # B4
        recv, gdown, dgrad = tr.buffers["recv"], tr.buffers["gdown"], tr.buffers["dgrad"]
        dgate, dup = gmm_dgrad_swiglu_bwd_raw(gdown, w_down, gate, up, off_local, True)
        # the down projection's weight gradient needs none of the GEMMs below: a side stream
        g_down, join = run_on_side(lambda: gmm_bwd_B_raw(h, w_down, off_local, gdown, True),
                                   grad_out.device)
        if dgrad_dual_ok(dgate, w_gate, dup, w_up):
            dgrad_dual_into(dgate, w_gate, dup, w_up, dgrad, off_local, tr.capacity, True)
        else:
            _gmm_call("moe_gmm_dgrad", dgate, w_gate, dgrad, off_local, tr.capacity,
                      w_gate.shape[1], w_gate.shape[2], El, True)
            dgrad_up = gmm_dgrad_raw(dup, w_up, off_local, True)
            _lib.check(lib.moe_add_rows(_lib.ptr(dgrad), _lib.ptr(dgrad_up),
                                        _lib.ptr(off_local[El:]), tr.capacity, d, dt, stream),
                       "moe_add_rows")
        g_gate = gmm_bwd_B_raw(recv, w_gate, off_local, dgate, True)
        g_up = gmm_bwd_B_raw(recv, w_up, off_local, dup, True)
        join()
        tr.barrier()                                               # B5
        grad_x = torch.empty(T, d, device=grad_out.device, dtype=grad_out.dtype)
        _lib.check(lib.moe_ep_combine(_lib.ptr(tr.bases["dgrad"]), dt, _lib.ptr(ranks), _lib.ptr(rows),
                                      None, 0, T, K, d, _lib.ptr(grad_x), _lib.ptr(status), stream),
                   "moe_ep_combine")
        _lib.count_launches(3)
        tr.pending_backward = False
        if hasattr(tr, "record_health") and not torch.cuda.is_current_stream_capturing():
            tr.record_health()
        return grad_x, grad_w, None, g_gate, g_up, g_down, None, None


def peer_experts(x, weights, indices, w_gate, w_up, w_down, transport: PeerTransport,
                 num_experts: int) -> torch.Tensor:
    """The EP expert segment over peer memory (differentiable in x, weights and the local
    expert weights): out[t] = sum_k weights[t,k] * expert_{indices[t,k]}(x[t])."""
    return _PeerExperts.apply(x, weights, indices, w_gate, w_up, w_down, transport, num_experts)


def capacity_rows(tokens_per_rank: int, top_k: int, world: int) -> int:
    """Receive-buffer rows for the worst case: every slot of every rank on one rank."""
    return tokens_per_rank * top_k * world
