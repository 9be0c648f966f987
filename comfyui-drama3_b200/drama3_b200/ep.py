"""Expert parallelism for the routed experts over the GPUs of one node (one process per GPU, torch.distributed):
rank r holds a contiguous block of the experts.

Decode (ExpertParallelDecode): every rank sees all rows (lines are replicated), runs the fused decode over its own
experts only and produces an fp32 partial [M, H]; the partials are gathered and summed in rank order, then rounded
to bf16 once, so every rank ends with the same output.

Prompt pass (ExpertParallelPrefill): every rank brings its own rows; each (row, rank) pair travels to the rank that
holds its expert and its output travels back (two all-to-alls), then each rank weights and sums its rows' pairs.

The reference runs on one GPU; this is the multi-GPU layout of its decode step (experts split, tokens replicated,
partial combines reduced). Two exchanges: an all-gather over NCCL (128 KB per layer at 16 lines), or PeerExchange,
where the decode kernel's combine stores its partial straight into every rank's exchange area over NVLink (P2P
stores through CUDA IPC mappings) and a small reduce kernel sums them once all ranks' flags are up - no collective
launch, the transfer overlapping the combine.
"""
import ctypes

import torch
import torch.distributed as dist

from . import _lib, kernels, offload

EP_MAX_RANKS = 8


class ExchangeStruct(ctypes.Structure):
    """The device struct the decode and reduce kernels read (d3::EpExchange)."""
    _fields_ = [("slots", ctypes.c_uint64 * EP_MAX_RANKS), ("flags", ctypes.c_uint64 * EP_MAX_RANKS),
                ("epoch", ctypes.c_uint64), ("world", ctypes.c_int32), ("rank", ctypes.c_int32),
                ("m_max", ctypes.c_int32), ("h", ctypes.c_int32)]


def exchange_layout(world, m_max, hidden):
    """(area bytes, flags offset): fp32 slots [2][world][m_max][hidden], then at the next 256-byte boundary the
    flags [2][8] (uint32) and this rank's call counter."""
    size = _lib.lib().d3_ep_exchange_bytes(world, m_max, hidden)
    if size == 0:
        raise ValueError(f"no exchange for world {world}, m_max {m_max}, hidden {hidden}")
    slots = 2 * world * m_max * hidden * 4
    return size, (slots + 255) // 256 * 256


def exchange_struct(slot_ptrs, flags_offset, rank, m_max, hidden):
    """The struct for this rank, from the base addresses of every rank's area as mapped here."""
    st = ExchangeStruct()
    for r, base in enumerate(slot_ptrs):
        st.slots[r] = base
        st.flags[r] = base + flags_offset
    st.epoch = slot_ptrs[rank] + flags_offset + 2 * EP_MAX_RANKS * 4
    st.world, st.rank, st.m_max, st.h = len(slot_ptrs), rank, m_max, hidden
    return bytes(st)


class PeerExchange:
    """Exchange areas for up to m_max lines of `hidden` columns, one per rank of `group` (one process per GPU of one
    node), each mapped into every other rank with CUDA IPC. Collective to create and to close. One exchange serves
    every layer: calls go through it one at a time, in the same order on every rank."""

    def __init__(self, m_max, hidden, device, group=None):
        self.group, self.m_max, self.hidden = group, m_max, hidden
        self.rank, self.world = dist.get_rank(group), dist.get_world_size(group)
        if self.world > EP_MAX_RANKS:
            raise ValueError(f"a peer exchange spans at most {EP_MAX_RANKS} ranks, not {self.world}")
        size, flags_offset = exchange_layout(self.world, m_max, hidden)
        self.area = torch.zeros((size,), dtype=torch.uint8, device=device)
        torch.cuda.synchronize(device)
        handle = (ctypes.c_char * 64)()
        offset = ctypes.c_size_t()
        with torch.cuda.device(self.area.device):
            _lib.check(_lib.lib().d3_ipc_handle(ctypes.c_void_p(self.area.data_ptr()), handle,
                                                ctypes.byref(offset)), "ipc_handle")
        handles = [None] * self.world
        dist.all_gather_object(handles, (bytes(handle), offset.value), group=group)
        self.bases, ptrs = [], []
        with torch.cuda.device(self.area.device):
            for r, (h, off) in enumerate(handles):
                if r == self.rank:
                    ptrs.append(self.area.data_ptr())
                    continue
                ptr, base = ctypes.c_void_p(), ctypes.c_void_p()
                _lib.check(_lib.lib().d3_ipc_open(h, off, ctypes.byref(ptr), ctypes.byref(base)), "ipc_open")
                self.bases.append(base.value)
                ptrs.append(ptr.value)
        raw = exchange_struct(ptrs, flags_offset, self.rank, m_max, hidden)
        self.device_struct = torch.frombuffer(bytearray(raw), dtype=torch.uint8).to(self.area.device)
        dist.barrier(group=group)

    def close(self):
        """Collective: unmap the peers' areas once every rank is done with them."""
        if self.bases is None:
            return
        torch.cuda.synchronize(self.area.device)
        dist.barrier(group=self.group)
        with torch.cuda.device(self.area.device):
            for base in self.bases:
                _lib.check(_lib.lib().d3_ipc_close(ctypes.c_void_p(base)), "ipc_close")
        self.bases = None
        dist.barrier(group=self.group)


def expert_range(num_experts, rank, world):
    """(first, count) of the contiguous block of experts rank `rank` of `world` holds: the blocks differ by at most
    one expert and cover [0, num_experts) in rank order."""
    base, extra = divmod(num_experts, world)
    first = rank * base + min(rank, extra)
    return first, base + (1 if rank < extra else 0)


def local_banks(banks, num_experts, rank, world):
    """This rank's slice of whole banks (gate_up, down) laid out [E * rows, ...]: every per-row field sliced by expert
    (fp8 128 x 128 block scales by blocks of rows)."""
    first, count = expert_range(num_experts, rank, world)
    out = []
    for bank in banks:
        sl = {}
        for name, t in bank.items():
            per = t.shape[0] // num_experts
            sl[name] = t[first * per:(first + count) * per]
        out.append(sl)
    return tuple(out)


def sum_in_rank_order(gathered):
    """gathered [world, M, H] fp32 -> [M, H] fp32: ((p0 + p1) + p2) + ..., the same on every rank."""
    out = gathered[0].clone()
    for r in range(1, gathered.shape[0]):
        out += gathered[r]
    return out


class ExpertParallelDecode:
    """The decode of one MoE layer with this rank's experts. `decode_fn(x, ids, weights) -> fp32 [M, H]` replaces
    the GPU kernel (kernels.moe_decode_ep over `banks`) when given, so the exchange can be exercised on CPU ranks.
    With `peer` (a PeerExchange) the partials cross NVLink inside the decode kernel instead of an NCCL all-gather."""

    def __init__(self, kind, banks, num_experts, group=None, codebooks=(None, None), decode_fn=None, peer=None):
        self.kind, self.banks, self.num_experts, self.group = kind, banks, num_experts, group
        self.codebooks, self.decode_fn, self.peer = codebooks, decode_fn, peer
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.e_first, self.e_count = expert_range(num_experts, self.rank, self.world)
        self.workspace = {}

    def _workspace(self, x, ids):
        key = (x.device, x.shape[0], ids.shape[-1])
        if key not in self.workspace:
            wkey = kernels._lib.WEIGHT_KEY[self.kind]
            e_local = self.banks[1][wkey].shape[0] // x.shape[1]
            inter = self.banks[0][wkey].shape[0] // (2 * e_local)
            self.workspace[key] = kernels.decode_workspace(x.shape[0], ids.shape[-1], inter, x.device)
        return self.workspace[key]

    def partial(self, x, ids, weights):
        if self.decode_fn is not None:
            return self.decode_fn(x, ids, weights)
        return kernels.moe_decode_ep(self.kind, x, ids, weights, self.banks, self.e_first, self.num_experts,
                                     self.codebooks, workspace=self._workspace(x, ids))

    def __call__(self, x, ids, weights):
        """[M, H] bfloat16, the same on every rank: the whole layer's decode of rows x [M, H] routed to ids [M, k]."""
        if self.peer is not None:
            M, H = x.shape
            if M > self.peer.m_max or H != self.peer.hidden:
                raise ValueError(f"[{M}, {H}] rows do not fit the peer exchange ({self.peer.m_max}, {self.peer.hidden})")
            kernels.moe_decode_ep(self.kind, x, ids, weights, self.banks, self.e_first, self.num_experts,
                                  self.codebooks, workspace=self._workspace(x, ids),
                                  exchange=self.peer.device_struct)
            return kernels.ep_reduce(self.peer.device_struct, M, H)
        part = self.partial(x, ids, weights).float().contiguous()
        gathered = torch.empty((self.world * part.shape[0], part.shape[1]), dtype=part.dtype, device=part.device)
        dist.all_gather_into_tensor(gathered, part, group=self.group)
        return sum_in_rank_order(gathered.view(self.world, *part.shape)).to(torch.bfloat16)


def expert_owner(ids, num_experts, world):
    """The rank holding each expert id under expert_range's blocks; -1 for ids outside [0, num_experts)."""
    base, extra = divmod(num_experts, world)
    big = extra * (base + 1)
    owner = torch.where(ids < big, ids // (base + 1), extra + (ids - big) // max(base, 1))
    return torch.where((ids >= 0) & (ids < num_experts), owner, torch.full_like(owner, -1))


def local_pairs(kind, banks, e_count, rows, codebooks, x, local_ids):
    """fp32 [R, rows[1]]: rows x [R, H] (bfloat16 or float32) each through its expert local_ids [R] (0-based in this
    rank's block of e_count experts, banks = local_banks), unweighted, in the given order: the two grouped GEMMs of
    the prompt pass over the rows sorted by expert on the device (offload.prefill_plan), then put back in order. Rows
    whose id is outside [0, e_count) (padding) are not computed: their output rows are unspecified."""
    if x.shape[0] == 0:
        return torch.zeros((0, rows[1]), dtype=torch.float32, device=x.device)
    if not (x.dtype in (torch.bfloat16, torch.float32) and kernels.grouped_mma_fits(rows[0], x.shape[1])
            and kernels.grouped_mma_fits(rows[1], rows[0] // 2)):
        raise ValueError("an expert-parallel prompt pass runs on the tensor-core kernels only (bfloat16 or float32 "
                         "rows, N % 128 == 0, K % 256 == 0)")
    order, pos, groups, tiles = offload.prefill_plan(local_ids.view(-1, 1), e_count, drop_invalid=True)
    rotated = kind in offload.ROTATED_KINDS
    hidden = kernels.grouped_mma(kind, x, groups, banks[0], codebooks[0], rows[0], tiles, row_index=order,
                                 rotate=rotated)
    out = kernels.grouped_mma(kind, hidden, groups, banks[1], codebooks[1], rows[1], tiles, rotate=rotated,
                              swiglu=True)
    return out[pos]


def _wire(t):
    """Rows as 32-bit words for the all-to-all (bfloat16 rows bit for bit, two values a word)."""
    return t.view(torch.int32) if t.dtype == torch.bfloat16 else t


class ExpertParallelPrefill:
    """One MoE layer's prompt pass with this rank's experts (banks = local_banks(..., rank, world); rows = (2I, H),
    the rows per expert of gate_up and down). Called on every rank with that rank's own rows x [T_r, H] and their
    routing topk_idx / topk_weight [T_r, k]: each (row, rank) pair is sent to the rank holding its expert (all-to-all
    of the rows and of their experts' indices within the receiver's block), runs there through the grouped GEMMs on
    the tensor cores, and its fp32 output is sent back (all-to-all); the rank then weights and sums its rows' pairs in
    rank order (kernels.prefill_combine). Every pair's output is computed alone and crosses exactly, so the result is
    bit for bit the one-GPU prompt pass of the same rows (offload.resident_prefill). Pairs whose id is outside
    [0, num_experts) add nothing.
    The split sizes of the all-to-alls are read back to the host once per call. With `capacity` (pairs a rank sends
    to each rank, at most; T_r * k always suffices) the exchanges move fixed blocks of that many rows instead, padded,
    and nothing is read back, so that the call can be captured in a CUDA graph; pairs beyond the capacity add nothing
    and are counted in `self.dropped` (a device tensor).
    `pairs_fn(x, ids) -> fp32 [R, H]` (global expert ids) and `combine_fn(pair_out [T_r * k, H], weights) -> [T_r, H]`
    replace the kernels when given, so that the exchange runs on CPU ranks."""

    def __init__(self, kind, banks, num_experts, rows, group=None, codebooks=(None, None), pairs_fn=None,
                 combine_fn=None, capacity=None):
        self.kind, self.banks, self.num_experts, self.rows, self.group = kind, banks, num_experts, rows, group
        self.codebooks, self.pairs_fn, self.combine_fn = codebooks, pairs_fn, combine_fn
        self.rank, self.world = dist.get_rank(group), dist.get_world_size(group)
        self.e_first, self.e_count = expert_range(num_experts, self.rank, self.world)
        self.firsts = [expert_range(num_experts, r, self.world)[0] for r in range(self.world)]
        self.capacity = capacity
        self.dropped = None
        self._firsts = {}

    def firsts_on(self, device):
        """Each rank's first expert as an int64 tensor on `device`, made on first use and kept: a call captured in a
        CUDA graph cannot copy it in from host memory."""
        device = torch.device(device)
        if device not in self._firsts:
            self._firsts[device] = torch.tensor(self.firsts, dtype=torch.int64, device=device)
        return self._firsts[device]

    def pairs(self, x, local_ids):
        if self.pairs_fn is not None:
            valid = local_ids >= 0
            if bool(valid.all()):
                return self.pairs_fn(x, local_ids.to(torch.int64) + self.e_first)
            out = torch.zeros((x.shape[0], self.rows[1]), dtype=torch.float32, device=x.device)
            if bool(valid.any()):
                out[valid] = self.pairs_fn(x[valid], local_ids[valid].to(torch.int64) + self.e_first)
            return out
        return local_pairs(self.kind, self.banks, self.e_count, self.rows, self.codebooks, x, local_ids)

    def _combine(self, x, pair_out, topk_weight):
        T, k = topk_weight.shape
        if self.combine_fn is not None:
            return self.combine_fn(pair_out, topk_weight)
        if T == 0:
            return torch.empty((0, self.rows[1]), dtype=x.dtype, device=x.device)
        pos = torch.arange(T * k, device=x.device).view(T, k)
        dtype = torch.float32 if x.dtype == torch.float32 else torch.bfloat16
        return kernels.prefill_combine(pair_out, pos, topk_weight, dtype=dtype).to(x.dtype)

    def _fixed(self, x, topk_idx, topk_weight):
        """The exchange in fixed blocks of `capacity` rows per rank pair: no host sync."""
        T, k = topk_idx.shape
        W, C, device = self.world, self.capacity, x.device
        flat = topk_idx.reshape(-1).to(torch.int64)
        owner = expert_owner(flat, self.num_experts, W)
        # each pair's rank among the pairs going to the same rank, by the device-side counting sort
        _, pos, groups, _ = offload.prefill_plan(owner.view(-1, 1), W)
        dest = torch.where(owner >= 0, owner, torch.full_like(owner, W))
        slot = pos - groups[:, 3].to(torch.int64)[dest]
        sent = (owner >= 0) & (slot < C)
        spill = W * C  # one extra row that pairs not sent write to, never sent
        index = torch.where(sent, owner * C + slot, torch.full_like(slot, spill))
        lost = ((owner >= 0) & (slot >= C)).sum()
        self.dropped = lost if self.dropped is None else self.dropped + lost
        firsts = self.firsts_on(device)
        send_x = torch.zeros((spill + 1, x.shape[1]), dtype=x.dtype, device=device)
        send_x[index] = x[torch.arange(T * k, device=device) // k]
        send_ids = torch.full((spill + 1,), -1, dtype=torch.int32, device=device)
        send_ids[index] = (flat - firsts[owner.clamp(min=0)]).to(torch.int32)
        wire = _wire(send_x[:spill])
        recv_x = torch.empty_like(wire)
        dist.all_to_all_single(recv_x, wire, group=self.group)
        recv_ids = torch.empty((spill,), dtype=torch.int32, device=device)
        dist.all_to_all_single(recv_ids, send_ids[:spill].contiguous(), group=self.group)
        if x.dtype == torch.bfloat16:
            recv_x = recv_x.view(torch.bfloat16)
        y = self.pairs(recv_x, recv_ids).to(torch.float32).contiguous()
        back = torch.empty((spill + 1, self.rows[1]), dtype=torch.float32, device=device)
        back[spill] = 0.0
        dist.all_to_all_single(back[:spill], y, group=self.group)
        return self._combine(x, back[index], topk_weight)

    def __call__(self, x, topk_idx, topk_weight):
        """[T_r, H] in x's dtype: this rank's rows through the whole layer's experts."""
        if self.capacity is not None:
            return self._fixed(x, topk_idx, topk_weight)
        T, k = topk_idx.shape
        device = x.device
        flat = topk_idx.reshape(-1)
        owner = expert_owner(flat, self.num_experts, self.world)
        dest = torch.where(owner >= 0, owner, torch.full_like(owner, self.world))
        order = torch.sort(dest, stable=True).indices
        counts = torch.bincount(dest, minlength=self.world + 1)[:self.world].contiguous()
        recv = torch.empty_like(counts)
        dist.all_to_all_single(recv, counts, group=self.group)
        send_counts, recv_counts = counts.tolist(), recv.tolist()
        n_send, n_recv = sum(send_counts), sum(recv_counts)
        sel = order[:n_send]
        firsts = self.firsts_on(device)
        send_ids = (flat[sel] - firsts[owner[sel]]).to(torch.int32)
        send_x = _wire(x[sel // k].contiguous())
        recv_x = torch.empty((n_recv, send_x.shape[1]), dtype=send_x.dtype, device=device)
        dist.all_to_all_single(recv_x, send_x, recv_counts, send_counts, group=self.group)
        recv_ids = torch.empty((n_recv,), dtype=torch.int32, device=device)
        dist.all_to_all_single(recv_ids, send_ids, recv_counts, send_counts, group=self.group)
        if x.dtype == torch.bfloat16:
            recv_x = recv_x.view(torch.bfloat16)
        y = self.pairs(recv_x, recv_ids).to(torch.float32).contiguous()
        back = torch.empty((n_send, self.rows[1]), dtype=torch.float32, device=device)
        dist.all_to_all_single(back, y, send_counts, recv_counts, group=self.group)
        pair_out = torch.zeros((T * k, self.rows[1]), dtype=torch.float32, device=device)
        pair_out[sel] = back
        return self._combine(x, pair_out, topk_weight)
