"""
KV-head sharding of the paged hot path across the GPUs of one node.

Attention and the KV write are independent per kv head, so N GPUs split the
kv heads: rank r owns kv heads ``[r*Hkv/N, (r+1)*Hkv/N)`` and the query heads
of their GQA groups, holds its own pool shard ``(blocks, 16, Hkv/N, D)`` with the
SAME block ids (block tables and slot mappings are replicated unchanged), runs
the write and the attention kernels on its shard, and the per-rank outputs are
all-gathered over NVLink with NCCL (``torch.distributed`` backend "nccl").

MemForge itself is single-device (``memforge_ml/runtime/continuous_engine.py:164``
takes one device); this module is the multi-GPU layer the B200 build adds.

The outputs are assembled one of two ways:

* ``gather_heads``: ``all_gather_into_tensor`` of the per-rank output
  ``[B, Hq/N, D]`` into ``[N*B, Hq/N, D]``, then one permute back to
  ``[B, Hq, D]``.  Every rank runs the same collectives in the same order.
* ``PeerOutput`` (decode batches): every rank's full ``[B, Hq, D]`` output is
  mapped into every other rank's process (CUDA IPC), the attention kernel stores
  its heads' rows straight into all of them over NVLink, and a flag barrier
  (``mf_peer_barrier``) completes the step.  No collective launch and no permute.
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Optional

import torch


@dataclass(frozen=True)
class HeadShard:
    """Which heads rank `rank` of `world` owns."""

    world: int
    rank: int
    num_q_heads: int
    num_kv_heads: int

    def __post_init__(self):
        if self.num_kv_heads % self.world:
            raise ValueError(f"{self.num_kv_heads} kv heads do not split over {self.world} GPUs")
        if self.num_q_heads % self.num_kv_heads:
            raise ValueError("query heads must be a multiple of kv heads")
        if not 0 <= self.rank < self.world:
            raise ValueError(f"rank {self.rank} outside world {self.world}")

    @property
    def kv_per_rank(self) -> int:
        return self.num_kv_heads // self.world

    @property
    def q_per_rank(self) -> int:
        return self.num_q_heads // self.world

    @property
    def kv_range(self):
        return self.rank * self.kv_per_rank, (self.rank + 1) * self.kv_per_rank

    @property
    def q_range(self):
        return self.rank * self.q_per_rank, (self.rank + 1) * self.q_per_rank

    def local_q(self, q: torch.Tensor) -> torch.Tensor:
        """This rank's query heads of ``[rows, Hq, D]`` (a view: no copy)."""
        a, b = self.q_range
        return q[:, a:b]

    def local_kv(self, kv: torch.Tensor) -> torch.Tensor:
        """This rank's kv heads of ``[rows, Hkv, D]`` new keys/values (a view)."""
        a, b = self.kv_range
        return kv[:, a:b]


def gather_heads(local_out: torch.Tensor, group=None,
                 out: Optional[torch.Tensor] = None,
                 staging: Optional[torch.Tensor] = None) -> torch.Tensor:
    """
    All-gather per-rank head slices ``[rows, Hq/N, D]`` into ``[rows, Hq, D]``.

    One ``all_gather_into_tensor`` into ``[N*rows, Hq/N, D]`` then a permute
    copy; pass ``staging``/``out`` to keep the step allocation-free (CUDA graphs).
    """
    import torch.distributed as dist
    world = dist.get_world_size(group)
    rows, hq_local, d = local_out.shape
    if staging is None:
        staging = torch.empty((world * rows, hq_local, d), dtype=local_out.dtype,
                              device=local_out.device)
    # Concatenated along dim 0 (the form both NCCL and gloo accept).
    dist.all_gather_into_tensor(staging.view(world * rows, hq_local, d), local_out.contiguous(),
                                group=group)
    full = staging.view(world, rows, hq_local, d).permute(1, 0, 2, 3).reshape(
        rows, world * hq_local, d)
    if out is None:
        return full
    out.copy_(full)
    return out


class PeerOutput:
    """
    The full ``[rows, Hq, D]`` decode output of a head-sharded step, held by
    every rank and written by all of them.

    Each rank allocates one arena holding ``buffers`` output tensors and a flag
    array of ``world`` int32, exports it through CUDA IPC (``mf_ipc_export``)
    and maps every peer's arena into its own device's address space
    (``mf_ipc_open``, with peer access enabled).  ``pointers(b)`` are the
    addresses of buffer ``b`` on all GPUs as this process sees them, for
    ``mf_attention_args.out_peers``; ``barrier()`` runs ``mf_peer_barrier`` with
    the next epoch.  Buffers alternate per step (``buffers`` of them, 2 by
    default).  The barrier of step i orders only each rank's own stream: once
    it completes, every rank has launched, on its stream, everything it queued
    before its step-i attention.  So the rule for callers is: every read of
    ``outs[b]`` (an o_proj, a copy to the host) must be stream-ordered on this
    rank's stream before the rank's next ``step_peer`` call.  Then the stores
    that peers make into buffer b two steps later cannot overtake it.  A reader
    on a side stream, or one that runs asynchronously past the next step, needs
    that stream joined first, or more buffers (``buffers=k`` keeps a buffer
    untouched for k-1 further steps).  Construction and ``close`` are
    collective (all ranks, same arguments).
    """

    def __init__(self, rows: int, num_q_heads: int, head_dim: int, dtype: torch.dtype,
                 device: torch.device, group=None, buffers: int = 2):
        import ctypes
        import torch.distributed as dist
        from . import _lib as L
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.group = group
        if self.world > L.MF_MAX_OUT_PEERS:
            raise ValueError(f"peer output serves at most {L.MF_MAX_OUT_PEERS} GPUs")
        self.device = device
        elt = torch.empty((), dtype=dtype).element_size()
        out_bytes = (rows * num_q_heads * head_dim * elt + 255) // 256 * 256
        flag_off = out_bytes * buffers
        total = flag_off + (self.world * 4 + 255) // 256 * 256
        self.arena = torch.zeros(total, dtype=torch.uint8, device=device)
        self.outs = [self.arena[b * out_bytes: b * out_bytes + rows * num_q_heads * head_dim * elt]
                     .view(dtype).view(rows, num_q_heads, head_dim) for b in range(buffers)]
        self.flags = self.arena[flag_off: flag_off + self.world * 4].view(torch.int32)
        torch.cuda.synchronize(device)
        lib = L.lib()
        handle = ctypes.create_string_buffer(L.MF_IPC_HANDLE_BYTES)
        offset = ctypes.c_uint64(0)
        with torch.cuda.device(device):
            L.check(lib.mf_ipc_export(ctypes.c_void_p(self.arena.data_ptr()), handle,
                                      ctypes.byref(offset)), "mf_ipc_export")
        everyone = [None] * self.world
        dist.all_gather_object(everyone, (handle.raw, offset.value), group=group)
        self._opened = []  # (address, offset) of every peer arena mapped here
        bases = []
        with torch.cuda.device(device):
            for p, (h, off) in enumerate(everyone):
                if p == self.rank:
                    bases.append(self.arena.data_ptr())
                    continue
                ptr = ctypes.c_void_p(0)
                L.check(lib.mf_ipc_open(ctypes.create_string_buffer(h, L.MF_IPC_HANDLE_BYTES),
                                        off, ctypes.byref(ptr)), "mf_ipc_open")
                self._opened.append((ptr.value, off))
                bases.append(ptr.value)
        self._ptrs = [[base + b * out_bytes for base in bases] for b in range(buffers)]
        self.flag_ptrs = [base + flag_off for base in bases]
        self.epoch = 0
        dist.barrier(group=group)  # every rank has mapped every peer before first use

    @property
    def current(self) -> int:
        """Buffer index the next step writes."""
        return (self.epoch + 1) % len(self.outs)

    def pointers(self, b: int):
        return self._ptrs[b]

    def barrier(self) -> torch.Tensor:
        """Complete the step that wrote ``self.outs[self.current]``; return it."""
        from . import _kernels as K
        b = self.current
        self.epoch += 1
        K.peer_barrier(self.flag_ptrs, self.rank, self.epoch, self.device)
        return self.outs[b]

    def close(self) -> None:
        """Unmap the peer arenas (collective: no rank may still write into them)."""
        import ctypes
        import torch.distributed as dist
        from . import _lib as L
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        with torch.cuda.device(self.device):
            for ptr, off in self._opened:
                L.check(L.lib().mf_ipc_close(ctypes.c_void_p(ptr), off), "mf_ipc_close")
        self._opened.clear()


class ShardedPagedDecode:
    """
    One layer's pool shard plus the sharded KV-write + decode step.

    ``key_pool``/``value_pool`` hold this rank's kv heads only:
    ``(num_blocks, 16, Hkv/N, D)``.  ``step`` takes the FULL new K/V
    ``[B, Hkv, D]`` and query ``[B, Hq, D]`` (each rank slices its heads as a
    view), writes the rank's heads of the new token into its shard, runs paged
    decode over its heads and returns the gathered ``[B, Hq, D]``.
    """

    def __init__(self, shard: HeadShard, num_blocks: int, head_dim: int,
                 dtype: torch.dtype = torch.bfloat16, device=None, block_size: int = 16,
                 group=None):
        self.shard = shard
        self.block_size = block_size
        self.head_dim = head_dim
        self.group = group
        device = device or torch.device("cuda", torch.cuda.current_device())
        shape = (num_blocks, block_size, shard.kv_per_rank, head_dim)
        self.key_pool = torch.zeros(shape, dtype=dtype, device=device)
        self.value_pool = torch.zeros(shape, dtype=dtype, device=device)
        self._local_out = None
        self._staging = None

    def write(self, new_k: torch.Tensor, new_v: torch.Tensor, slots: torch.Tensor) -> None:
        from . import _kernels as K
        K.reshape_and_cache(self.shard.local_kv(new_k), self.shard.local_kv(new_v),
                            self.key_pool, self.value_pool, slots)

    def attend(self, q: torch.Tensor, block_tables: torch.Tensor, kv_lens: torch.Tensor,
               scale: Optional[float] = None) -> torch.Tensor:
        """This rank's heads of the decode output, ``[B, Hq/N, D]``."""
        from . import _kernels as K
        rows = q.shape[0]
        if self._local_out is None or self._local_out.shape[0] != rows:
            self._local_out = torch.empty((rows, self.shard.q_per_rank, self.head_dim),
                                          dtype=q.dtype, device=q.device)
            self._staging = torch.empty((self.shard.world * rows, self.shard.q_per_rank,
                                         self.head_dim), dtype=q.dtype, device=q.device)
        scale = scale if scale is not None else 1.0 / math.sqrt(self.head_dim)
        K.paged_attention(self.shard.local_q(q), self._local_out, self.key_pool, self.value_pool,
                          block_tables, kv_lens, q_per_seq=1, scale=scale, causal=True)
        return self._local_out

    def step(self, q, new_k, new_v, slots, block_tables, kv_lens, scale=None,
             out: Optional[torch.Tensor] = None) -> torch.Tensor:
        self.write(new_k, new_v, slots)
        local = self.attend(q, block_tables, kv_lens, scale)
        if self.shard.world == 1:
            return local if out is None else out.copy_(local)
        return gather_heads(local, self.group, out=out, staging=self._staging)

    def step_peer(self, peer: PeerOutput, q, new_k, new_v, slots, block_tables, kv_lens,
                  scale=None) -> torch.Tensor:
        """
        The same step with the outputs assembled over peer memory: returns the full
        ``[B, Hq, D]`` (one of ``peer``'s buffers, valid until the step after next).
        """
        from . import _kernels as K
        self.write(new_k, new_v, slots)
        b = peer.current
        scale = scale if scale is not None else 1.0 / math.sqrt(self.head_dim)
        K.paged_attention(self.shard.local_q(q), peer.outs[b], self.key_pool, self.value_pool,
                          block_tables, kv_lens, q_per_seq=1, scale=scale, causal=True,
                          out_peers=peer.pointers(b),
                          out_head_offset=self.shard.q_range[0])
        return peer.barrier()
