"""Multi-GPU placement of the hot path: one process per GPU, no collective inside a decode step except the output
gather of KV-head sharding.

The reference has no multi-GPU code of its own (tensor parallelism comes from vLLM, kushkash README "Tensor
parallel"); decode work units (sequence, kv head, split) and quantize-on-write units (sequence, page, head) are
independent, so they shard without communication:

  request partitioning  rank r owns whole sequences (their pages, block-table rows and tail slots); a step needs no
                        collective.  partition_requests balances the ranks by cached tokens (the decode's bytes).
  kv-head partitioning  for a few very long sequences: rank r owns kv heads [h0, h1) of every
                        sequence and the q heads h0*G .. h1*G; after the local split-KV decode, the [S, Hq/N, D]
                        outputs are gathered into [S, Hq, D] on every rank -- the only data-path exchange.  Two
                        forms: gather_heads (an NCCL all_gather) and PeerGather / decode_gathered, where the
                        split-KV combine itself stores every rank's slice into every rank's buffer over NVLink (CUDA
                        IPC mappings) and a bounded wait kernel completes it: no library collective in the step,
                        which then captures in one CUDA graph.
"""
from __future__ import annotations

import heapq

import torch


def partition_requests(seq_lens: list[int], world: int) -> list[list[int]]:
    """Sequence indices per rank, balanced by cached tokens (longest first onto the least-loaded rank; ties by rank,
    so every rank computes the same assignment)."""
    if world < 1:
        raise ValueError("world must be >= 1")
    heap = [(0, r) for r in range(world)]
    out: list[list[int]] = [[] for _ in range(world)]
    for i in sorted(range(len(seq_lens)), key=lambda i: (-seq_lens[i], i)):
        load, r = heapq.heappop(heap)
        out[r].append(i)
        heapq.heappush(heap, (load + int(seq_lens[i]), r))
    return [sorted(x) for x in out]


def kv_head_range(num_kv_heads: int, rank: int, world: int) -> tuple[int, int]:
    """[h0, h1) of the kv heads rank `rank` owns; heads must divide evenly (8 kv heads over 1, 2, 4 or 8 GPUs)."""
    if num_kv_heads % world:
        raise ValueError(f"{num_kv_heads} kv heads do not split over {world} ranks")
    per = num_kv_heads // world
    return rank * per, (rank + 1) * per


def gather_heads(local_out: torch.Tensor, group=None) -> torch.Tensor:
    """[S, Hq/N, D] outputs of this rank's q heads -> [S, Hq, D] on every rank (all_gather over the process group:
    NCCL over NVLink on GPUs, gloo on CPU), heads in rank order."""
    import torch.distributed as dist
    world = dist.get_world_size(group)
    if world == 1:
        return local_out
    parts = [torch.empty_like(local_out) for _ in range(world)]
    dist.all_gather(parts, local_out.contiguous(), group=group)
    return torch.cat(parts, dim=1)


class _DeviceArray:
    """A raw device allocation seen through __cuda_array_interface__ (torch.as_tensor maps it without a copy)."""

    def __init__(self, ptr: int, shape: tuple[int, ...], typestr: str):
        self.__cuda_array_interface__ = {"shape": shape, "typestr": typestr, "data": (ptr, False), "version": 3,
                                         "strides": None}


class PeerGather:
    """Gathered [S, Hq, D] decode outputs of KV-head sharding through peer memory, in place of gather_heads.

    Each rank's split-KV combine (kush_sm100_combine_gather) stores its q heads into every rank's buffer over
    NVLink and then signals the peers; `wait()` (kush_sm100_gather_wait, a bounded one-warp wait) makes the buffer
    complete for what follows on the stream.  Neither is a library collective, so a step that uses them captures in
    one CUDA graph.  `slots` buffers (one per layer, say) live in one CUDA-IPC allocation per rank, mapped by every
    other rank at construction (a collective call: all ranks construct together; the handles travel over the
    process group).  Every rank must then make the same sequence of gathers.  Without an initialised process group
    (or with one rank) the gather is local.  `close()` unmaps and frees (the tensors in `outs` die with it).

    Slot reuse.  A wait only proves that every rank has stored the current gather; it says nothing about whether a
    peer still reads a slot that another gather is about to fill.  What orders a peer's stores: its combine of gather
    g runs after its wait of gather g - 1, which returns once every rank has run its own combine of gather g - 1.  So
    with gathers filling slots round robin, a rank's reads of the slot that gather g filled (a copy of the outputs,
    the next layer's kernels) must be stream-ordered before its own combine of gather g + slots - 1.  One slot per
    layer and the outputs read after the whole step break this for every layer but the last; give each step its own
    set of slots (2 x layers, alternating per step) or copy each output out right after its wait."""

    def __init__(self, n_seqs: int, num_q_heads: int, head_dim: int, dtype: torch.dtype, slots: int = 1,
                 group=None):
        import torch.distributed as dist
        from . import _cuda
        self._cuda, self.group = _cuda, group
        dist_on = dist.is_available() and dist.is_initialized()
        self.world = dist.get_world_size(group) if dist_on else 1
        self.rank = dist.get_rank(group) if dist_on else 0
        if self.world > 32:
            raise ValueError("PeerGather supports up to 32 ranks")
        if num_q_heads % self.world:
            raise ValueError(f"{num_q_heads} q heads do not split over {self.world} ranks")
        self.shape, self.dtype, self.slots = (n_seqs, num_q_heads, head_dim), dtype, slots
        esize = torch.empty(0, dtype=dtype).element_size()
        self.slot_bytes = -(-n_seqs * num_q_heads * head_dim * esize // 256) * 256
        self.flags_off = slots * self.slot_bytes                 # [world] uint32 gather counts written by the ranks
        self.ctr_off = self.flags_off + 256                      # [2] uint32: finished blocks, own gather count
        self.device = torch.device("cuda", torch.cuda.current_device())
        self.base = _cuda.ipc_alloc(self.ctr_off + 256)
        self.peers = [self.base]
        if self.world > 1:
            handles: list = [None] * self.world
            dist.all_gather_object(handles, _cuda.ipc_handle(self.base), group=group)
            self.peers = [self.base if r == self.rank else _cuda.ipc_open(handles[r]) for r in range(self.world)]
        self.out_tab = torch.tensor([[p + s * self.slot_bytes for p in self.peers] for s in range(slots)],
                                    dtype=torch.int64, device=self.device)
        self.flag_tab = torch.tensor([p + self.flags_off for p in self.peers], dtype=torch.int64, device=self.device)
        itype = {1: "|u1", 2: "<i2", 4: "<i4"}[esize]
        n = n_seqs * num_q_heads * head_dim
        self.outs = [torch.as_tensor(_DeviceArray(self.base + s * self.slot_bytes, (n,), itype), device=self.device)
                     .view(dtype).view(n_seqs, num_q_heads, head_dim) for s in range(slots)]
        self.count = torch.as_tensor(_DeviceArray(self.base + self.ctr_off, (2,), "<i4"), device=self.device)
        if self.world > 1:
            dist.barrier(group=group)

    def combine(self, ops, part_ml: int, part_o: int, n_splits: int, hkv: int, n_seqs: int, slot: int = 0) -> None:
        """The split-KV combine of this rank's `hkv` kv heads, stored into slot `slot` of every rank."""
        c = ops.cfg
        if not 0 <= slot < self.slots:
            raise ValueError(f"slot {slot} out of range ({self.slots} slots)")
        if (n_seqs, hkv * c.group * self.world, c.head_dim) != self.shape:
            raise ValueError(f"combine of [{n_seqs}, {hkv}x{c.group}, {c.head_dim}] does not fit {self.shape}")
        self._cuda.check(self._cuda.lib().kush_sm100_combine_gather(
            c.head_dim, c.dtype_code, c.group, self.out_tab[slot].data_ptr(), self.rank, self.world, part_ml, part_o,
            n_splits, hkv, n_seqs, self.flag_tab.data_ptr(), self.base + self.ctr_off,
            self._cuda.raw_stream(self.device.index)), "kush_sm100_combine_gather")

    def wait(self) -> None:
        """Wait (on the stream) until every rank's stores of the latest gather have arrived."""
        self._cuda.check(self._cuda.lib().kush_sm100_gather_wait(
            self.base + self.flags_off, self.world, self.base + self.ctr_off,
            self._cuda.raw_stream(self.device.index)), "kush_sm100_gather_wait")

    def close(self) -> None:
        import torch.distributed as dist
        if self.base is None:
            return
        torch.cuda.synchronize(self.device)
        if self.world > 1:
            dist.barrier(group=self.group)                       # no rank still stores into a mapping being closed
            for r, p in enumerate(self.peers):
                if r != self.rank:
                    self._cuda.ipc_close(p)
            dist.barrier(group=self.group)
        self._cuda.ipc_free(self.base)
        self.base, self.outs = None, []


def decode_gathered(ops, q: torch.Tensor, cache: torch.Tensor, block_table: torch.Tensor, seq_lens: torch.Tensor,
                    tail_idx: torch.Tensor, tail_k: torch.Tensor, scale: float, n_splits: int, work: torch.Tensor,
                    gather: PeerGather, slot: int = 0) -> torch.Tensor:
    """Ops.decode of this rank's kv heads with the outputs of all ranks gathered into gather.outs[slot]: the split-KV
    decode (n_splits >= 2, `work` sized for it), the combine that stores into every rank, the wait for the peers."""
    part_ml, part_o = ops.decode_partials(q, cache, block_table, seq_lens, tail_idx, tail_k, scale, n_splits, work)
    gather.combine(ops, part_ml, part_o, n_splits, tail_k.shape[1], q.shape[0], slot)
    gather.wait()
    return gather.outs[slot]
