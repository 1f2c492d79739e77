"""Expert-parallel dispatch and combine of the MoE prologue across ranks (one process per GPU).

Rank r of N owns experts [r*E/N, (r+1)*E/N) (48 per GPU for E = 384 on 8 GPUs) and routes
its own tokens.  The path needs one exchange step per direction:

  dispatch  1. local router + expert maps over all E experts: the permuted rows are sorted
               by expert, hence already grouped by owner rank
            2. all-gather of the per-expert counts [E] -> [N, E]; every rank derives the send
               and receive splits from it, with no further round trip
            3. the routed rows go to their owners, where they end up grouped by local
               expert (then by sender, then in the sender's order): contiguous per-expert
               segments and their offsets, ready for the expert GEMMs
  combine   4. the owner sends the expert outputs back to the senders' permuted positions,
               and every sender finalizes its tokens: out[t] = sum_k w[t, k] * row(u2p[k*T + t])

Two implementations with the same row order and bit-identical results:

  PeerExpertParallel  the B200 path.  Steps 2-4 are libkolibri_b200 kernels that store into
                      the peers' exchange buffers (CUDA IPC mappings over NVLink / NVSwitch):
                      kb_router_maps_allgather (router + maps with the count all-gather in the
                      same kernel's tail), kb_ep_dispatch (the expansion, the pack and the
                      all-to-all in one pass: every row is written once, at its final grouped
                      row on the owner) and kb_ep_combine (return trip + finalize).  Nothing
                      synchronises with the host, so a layer can be captured in a CUDA graph.
  ExpertParallel      the same exchange as torch.distributed collectives (all_gather of the
                      counts, all_to_all_single of rows and metadata, a regrouping by local
                      expert on the owner).  all_to_all_single needs its splits on the host,
                      so it reads them back once per dispatch.  It runs on any backend, which
                      is how the exchange logic is tested on CPU ranks (gloo), and it is the
                      cross-check of the peer path on GPUs.

The reference repository runs on one GPU and has no such path; the layout follows the
(expert, token, slot) order of its maps (kernels/cuda/customKolibriBuildExpertMapsKernel.cu:
96-156) and its finalize (benchmarks/11_profile_2block_e2e.py:259-262).

ExpertParallel's local steps go through a `LocalOps` object.  The default one calls the
libkolibri_b200 kernels (CUDA tensors only, no fallback); the CPU tests of the exchange logic
substitute CPU implementations of the same four operations.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import torch
import torch.distributed as dist


class LocalOps:
    """The four local operations of the path, on the libkolibri_b200 kernels."""

    def router_maps(self, logits, bias, k):
        from . import ops
        ids, w, counts, offsets, p2u, u2p = ops.router_maps(logits, bias, k=k)
        return ids, w, counts, offsets, p2u, u2p

    def expert_maps(self, ids, num_experts):
        from . import ops
        return ops.expert_maps(ids, num_experts)

    def expand_rows(self, x, p2u):
        from . import ops
        return ops.expand_rows(x, p2u)

    def finalize(self, rows, u2p, w):
        from . import ops
        return ops.moe_finalize(rows, u2p, w)


@dataclass
class Dispatched:
    """What dispatch() returns: the sender-side state for combine() and the owner's rows."""
    # sender side
    T: int
    ids: torch.Tensor          # int32 [T, K] routed experts (global ids)
    weights: torch.Tensor      # fp32 [T, K]
    u2p: torch.Tensor          # int32 [K*T] local unpermuted -> permuted row
    send_splits: list          # rows sent to each rank
    recv_splits: list          # rows received from each rank
    # owner side
    rows: torch.Tensor         # [R, H] received rows grouped by local expert
    expert_offsets: torch.Tensor  # int64 [E/N + 1] segments of `rows` per local expert
    meta: torch.Tensor         # int32 [R, 3] received (expert, weight bits, origin), sender order
    group_p2u: torch.Tensor    # int32 [R] grouped position -> received row
    group_u2p: torch.Tensor    # int32 [R] received row -> grouped position


class ExpertParallel:
    """Dispatch/combine for one MoE layer with E experts and top-K routing over `group`."""

    def __init__(self, num_experts: int = 384, top_k: int = 6,
                 group: Optional[dist.ProcessGroup] = None, local_ops: Optional[LocalOps] = None):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if num_experts % self.world:
            raise ValueError("num_experts must be a multiple of the world size")
        self.E, self.K = num_experts, top_k
        self.Er = num_experts // self.world
        self.ops = local_ops or LocalOps()

    # ------------------------------------------------------------------------------------
    def dispatch(self, x: torch.Tensor, logits: torch.Tensor,
                 bias: Optional[torch.Tensor] = None) -> Dispatched:
        T, H = x.shape
        N, Er, K = self.world, self.Er, self.K
        ids, w, counts, offsets, p2u, u2p = self.ops.router_maps(logits, bias, K)
        permuted = self.ops.expand_rows(x, p2u)                   # [T*K, H], expert order
        # metadata of every permuted row: expert, weight bits, origin (slot*T + token)
        p2u_l = p2u.long()
        tok, slot = p2u_l % T, p2u_l // T
        flat = tok * K + slot
        meta = torch.stack([ids.reshape(-1)[flat].int(),
                            w.reshape(-1)[flat].contiguous().view(torch.int32),
                            p2u.int()], dim=1).contiguous()
        # counts of every rank, then the splits of both directions
        counts_all = torch.empty(N * self.E, dtype=counts.dtype, device=counts.device)
        dist.all_gather_into_tensor(counts_all, counts.contiguous(), group=self.group)
        per_owner = counts_all.view(N, N, Er).sum(-1).cpu()       # [sender, owner]
        send_splits = per_owner[self.rank].tolist()
        recv_splits = per_owner[:, self.rank].tolist()
        R = int(sum(recv_splits))
        recv_rows = torch.empty(R, H, dtype=x.dtype, device=x.device)
        recv_meta = torch.empty(R, 3, dtype=torch.int32, device=x.device)
        dist.all_to_all_single(recv_rows, permuted, recv_splits, send_splits, group=self.group)
        dist.all_to_all_single(recv_meta, meta, recv_splits, send_splits, group=self.group)
        # group the received rows by local expert (stable: sender, then sender's order)
        local_ids = (recv_meta[:, 0] - self.rank * Er).contiguous().view(R, 1)
        if R:
            _, loff, gp2u, gu2p = self.ops.expert_maps(local_ids, Er)
            rows = self.ops.expand_rows(recv_rows, gp2u)
        else:
            loff = torch.zeros(Er + 1, dtype=torch.int64, device=x.device)
            gp2u = torch.empty(0, dtype=torch.int32, device=x.device)
            gu2p = torch.empty(0, dtype=torch.int32, device=x.device)
            rows = recv_rows
        return Dispatched(T=T, ids=ids, weights=w, u2p=u2p, send_splits=send_splits,
                          recv_splits=recv_splits, rows=rows, expert_offsets=loff,
                          meta=recv_meta, group_p2u=gp2u, group_u2p=gu2p)

    def combine(self, d: Dispatched, expert_out: torch.Tensor) -> torch.Tensor:
        """expert_out: [R, H] outputs of the local experts in the grouped order of d.rows."""
        R, H = expert_out.shape
        back_rows = (self.ops.expand_rows(expert_out, d.group_u2p) if R
                     else expert_out)                             # received (sender) order
        mine = torch.empty(d.T * self.K, H, dtype=expert_out.dtype, device=expert_out.device)
        dist.all_to_all_single(mine, back_rows.contiguous(), d.send_splits, d.recv_splits,
                               group=self.group)
        return self.ops.finalize(mine, d.u2p, d.weights)


# ----------------------------------------------------------------------------------------
# The exchange on peer memory (kb_ep_* kernels): no NCCL call, no host round trip.
# ----------------------------------------------------------------------------------------
class _DeviceRows:
    """Zero-copy torch view of library-owned device memory (__cuda_array_interface__)."""

    def __init__(self, ptr: int, rows: int, cols: int, typestr: str):
        self.__cuda_array_interface__ = {"shape": (rows, cols), "typestr": typestr,
                                         "data": (ptr, False), "version": 3, "strides": None}


_VIEW = {torch.bfloat16: ("<i2", torch.int16), torch.float16: ("<f2", torch.float16),
         torch.float32: ("<f4", torch.float32)}


class PeerGroup:
    """The ranks' exchange buffers (kb_ep_alloc), each mapped into every rank through CUDA
    IPC: the kb_ep_group_t the kb_ep_* calls take.  One process per GPU of one node; the
    handles and the shape parameters are exchanged once over `group` (any backend).

    Collective to build and to close(): every rank of `group` makes the same calls."""

    def __init__(self, num_experts: int, top_k: int, max_tokens: int, row_bytes: int,
                 group: Optional[dist.ProcessGroup] = None,
                 device: Optional[torch.device] = None):
        import ctypes
        from . import _lib
        self._lib = lib = _lib.load()
        self.group = group
        on = dist.is_available() and dist.is_initialized()
        self.world = dist.get_world_size(group) if on else 1
        self.rank = dist.get_rank(group) if on else 0
        if self.world > _lib.KB_MAX_RANKS:
            raise ValueError(f"at most {_lib.KB_MAX_RANKS} ranks")
        self.device = torch.device(device or torch.device("cuda", torch.cuda.current_device()))
        self.E, self.K = int(num_experts), int(top_k)
        self.max_tokens, self.row_bytes = int(max_tokens), int(row_bytes)
        nbytes = int(lib.kb_ep_buffer_bytes(self.world, self.E, self.K, self.max_tokens,
                                            self.row_bytes))
        if nbytes == 0:
            raise ValueError("invalid exchange-buffer shape")
        own = ctypes.c_void_p()
        with torch.cuda.device(self.device):
            _lib.check(lib.kb_ep_alloc(nbytes, ctypes.byref(own)), "kb_ep_alloc")
        self._own, self._imported, self.nbytes = own.value, [], nbytes
        bufs = [0] * self.world
        bufs[self.rank] = own.value
        if self.world > 1:
            handle = (ctypes.c_uint8 * _lib.KB_IPC_HANDLE_BYTES)()
            _lib.check(lib.kb_ipc_export(own, handle), "kb_ipc_export")
            meta = torch.tensor([self.E, self.K, self.max_tokens, self.row_bytes, nbytes],
                                dtype=torch.int64)
            mine = torch.cat([torch.tensor(list(bytes(handle)), dtype=torch.int64), meta])
            comm_dev = self.device if dist.get_backend(group) == "nccl" else torch.device("cpu")
            allv = torch.empty(self.world, mine.numel(), dtype=torch.int64, device=comm_dev)
            dist.all_gather_into_tensor(allv, mine.to(comm_dev), group=group)
            allv = allv.cpu()
            if not bool((allv[:, -5:] == meta).all()):
                self._free()
                raise ValueError("ranks disagree on the exchange-buffer shape")
            with torch.cuda.device(self.device):
                for q in range(self.world):
                    if q == self.rank:
                        continue
                    h = (ctypes.c_uint8 * _lib.KB_IPC_HANDLE_BYTES)(
                        *[int(v) for v in allv[q, :_lib.KB_IPC_HANDLE_BYTES]])
                    ptr = ctypes.c_void_p()
                    _lib.check(lib.kb_ipc_import(h, ctypes.byref(ptr)), "kb_ipc_import")
                    self._imported.append(ptr.value)
                    bufs[q] = ptr.value
        arr = (ctypes.c_void_p * _lib.KB_MAX_RANKS)(*(bufs + [None] * (_lib.KB_MAX_RANKS - self.world)))
        self.desc = _lib.EpGroup(self.world, self.rank, self.E, self.K, self.max_tokens,
                                 self.row_bytes, arr)
        self.addr = ctypes.addressof(self.desc)

    def recv_rows(self, dtype: torch.dtype) -> torch.Tensor:
        """This rank's received-rows area as a [N*max_tokens*K, H] tensor (no copy)."""
        import ctypes
        from . import _lib
        ptr = ctypes.c_void_p()
        _lib.check(self._lib.kb_ep_recv_rows(self.addr, ctypes.byref(ptr)), "kb_ep_recv_rows")
        typestr, tdt = _VIEW[dtype]
        esize = torch.tensor([], dtype=dtype).element_size()
        cap = self.world * self.max_tokens * self.K
        t = torch.as_tensor(_DeviceRows(ptr.value, cap, self.row_bytes // esize, typestr),
                            device=self.device)
        return t.view(dtype) if tdt != dtype else t

    def barrier(self, stream: Optional[torch.cuda.Stream] = None) -> None:
        """Device-side barrier (kb_ep_barrier) on `stream`: the work queued after it starts on
        every rank together."""
        from . import _lib
        st = stream or torch.cuda.current_stream(self.device)
        _lib.check(self._lib.kb_ep_barrier(self.addr, st.cuda_stream), "kb_ep_barrier")

    def status(self) -> int:
        """The error word of this rank's buffer (0 clean, 1 timeout, 3 capacity)."""
        import ctypes
        from . import _lib
        out = ctypes.c_int(-1)
        with torch.cuda.device(self.device):
            _lib.check(self._lib.kb_workspace_status(
                self._own, _lib.KB_WS_EP, ctypes.byref(out),
                torch.cuda.current_stream(self.device).cuda_stream), "kb_workspace_status")
        return out.value

    def _free(self):
        if self._own:
            self._lib.kb_ep_free(self._own)
            self._own = None

    def close(self) -> None:
        """Unmap the peers' buffers and free this rank's (collective)."""
        if self._own is None:
            return
        torch.cuda.synchronize(self.device)
        if self.world > 1:
            dist.barrier(group=self.group)
        with torch.cuda.device(self.device):
            for p in self._imported:
                self._lib.kb_ipc_close(p)
            self._imported = []
            if self.world > 1:
                dist.barrier(group=self.group)
            self._free()


@dataclass
class PeerDispatched:
    """What PeerExpertParallel.dispatch returns (device tensors only)."""
    T: int
    ids: torch.Tensor             # int32 [T, K] routed experts (global ids)
    weights: torch.Tensor         # fp32 [T, K]
    u2p: torch.Tensor             # int32 [K*T]
    gathered: torch.Tensor        # int32 [N, E] every rank's per-expert counts
    rows: torch.Tensor            # [N*max_tokens*K, H] received rows, grouped by local expert
    expert_offsets: torch.Tensor  # int64 [E/N + 1] segments of `rows` (first [-1] rows valid)

    def num_rows(self) -> int:
        """Received rows (reads expert_offsets[-1]: synchronises with the stream)."""
        return int(self.expert_offsets[-1].item())


class PeerExpertParallel:
    """Dispatch/combine of one MoE layer over peer memory: the count all-gather, the row
    exchange and the return trip are libkolibri_b200 kernels that store straight into the
    owners' (and back into the senders') exchange buffers.  Same row order as
    ExpertParallel; nothing synchronises with the host, so a whole layer can be captured in a
    CUDA graph.  Every rank calls dispatch and combine in the same order."""

    def __init__(self, num_experts: int = 384, top_k: int = 6, hidden: int = 6144,
                 dtype: torch.dtype = torch.bfloat16, max_tokens: int = 4096,
                 group: Optional[dist.ProcessGroup] = None,
                 device: Optional[torch.device] = None):
        from . import _lib
        if dtype not in _VIEW:
            raise ValueError("dtype must be bfloat16, float16 or float32")
        esize = torch.tensor([], dtype=dtype).element_size()
        self.pg = PeerGroup(num_experts, top_k, max_tokens, hidden * esize, group, device)
        self.world, self.rank = self.pg.world, self.pg.rank
        self.E, self.K, self.H, self.dtype = num_experts, top_k, hidden, dtype
        self.Er = num_experts // self.world
        dev = self.pg.device
        self.gathered = torch.empty(self.world, num_experts, dtype=torch.int32, device=dev)
        self.recv_offsets = torch.empty(self.Er + 1, dtype=torch.int64, device=dev)
        self.rows = self.pg.recv_rows(dtype)
        self._dtype_code = {torch.bfloat16: _lib.KB_BF16, torch.float16: _lib.KB_F16,
                            torch.float32: _lib.KB_F32}[dtype]

    def counts_allgather(self, counts: torch.Tensor) -> torch.Tensor:
        from . import _lib
        _lib.check(self.pg._lib.kb_ep_counts_allgather(
            self.pg.addr, counts.data_ptr(), self.gathered.data_ptr(),
            torch.cuda.current_stream(counts.device).cuda_stream), "kb_ep_counts_allgather")
        return self.gathered

    def dispatch(self, x: torch.Tensor, logits: torch.Tensor,
                 bias: Optional[torch.Tensor] = None) -> PeerDispatched:
        from . import _lib, ops
        T = x.shape[0]
        if x.dtype != self.dtype or x.shape[1] != self.H or not x.is_contiguous():
            raise ValueError("x must be a contiguous [T, hidden] tensor of the group's dtype")
        if logits.shape[1] != self.E:
            raise ValueError(f"logits must have {self.E} columns")
        ids, w, counts, offsets, p2u, u2p = ops.router_maps_allgather(
            self.pg.addr, logits, bias, self.gathered, k=self.K)
        _lib.check(self.pg._lib.kb_ep_dispatch(
            self.pg.addr, x.data_ptr(), T, p2u.data_ptr(), self.gathered.data_ptr(),
            self.recv_offsets.data_ptr(), torch.cuda.current_stream(x.device).cuda_stream),
            "kb_ep_dispatch")
        return PeerDispatched(T=T, ids=ids, weights=w, u2p=u2p, gathered=self.gathered,
                              rows=self.rows, expert_offsets=self.recv_offsets)

    def combine(self, d: PeerDispatched, expert_out: torch.Tensor,
                out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """expert_out: the local experts' outputs in the grouped order of d.rows (it may be
        d.rows itself).  Returns out [T, H] = sum_k w[t, k] * expert row of (t, k)."""
        from . import _lib
        if out is None:
            out = torch.empty(d.T, self.H, dtype=self.dtype, device=expert_out.device)
        _lib.check(self.pg._lib.kb_ep_combine(
            self.pg.addr, expert_out.data_ptr(), d.gathered.data_ptr(), d.T, d.u2p.data_ptr(),
            d.weights.data_ptr(), out.data_ptr(), self._dtype_code,
            torch.cuda.current_stream(expert_out.device).cuda_stream), "kb_ep_combine")
        return out

    def close(self) -> None:
        self.pg.close()
