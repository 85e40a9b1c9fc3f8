"""
CUDA-graphed batched decode over the paged pool, with attention and KV writes
served by the sm_100a kernels.  B200 edition of
``memforge_ml/runtime/graphed_paged_decode.py``'s ``GraphedPagedDecoder``.

One decode step for up to ``max_batch`` sequences (one new token each) is the
model's whole forward: per layer the new token's K/V are written at its slot
(``mf_reshape_and_cache``, slots computed on the device from the block tables
and positions) and attention reads the context straight from the pool pages
(``mf_paged_attention``, context lengths read from the device).  Everything that
varies between steps (tokens, positions, block tables, lengths) is a device
tensor, so one captured graph per batch bucket serves every context length: no
context bucketing and no gather, unlike the reference's ``gather`` kernel
option.  Batches are padded to a power of two by repeating row 0; the
duplicate row writes identical values to the same slot and its logits are
dropped.

``attn_kernel`` accepts ``"sm100"`` only (the reference's ``"gather"`` and
``"triton"`` options name paths this build replaces).  The model runs with
the ``memforge_paged`` attention function for the graphed step only; its own
setting is restored afterwards.
"""

from __future__ import annotations

from contextlib import contextmanager
from typing import Dict, Optional, Sequence

import torch
from transformers.cache_utils import Cache, CacheLayerMixin

from . import _kernels as K
from . import attention_backend as AB


class _GraphLayer(CacheLayerMixin):
    """Cache layer of the graphed step: writes the new token, returns it unchanged."""

    is_sliding = False
    is_compileable = False

    def __init__(self, owner: "GraphedPagedDecoder", layer_idx: int):
        super().__init__()
        self.owner, self.layer_idx = owner, layer_idx
        self.is_initialized = True

    def update(self, key_states, value_states, *args, **kwargs):
        o, l = self.owner, self.layer_idx
        b = o._b
        # (B, H, 1, D) -> (B, H, D) rows at each row's slot, this layer's pool
        K.reshape_and_cache(key_states[:, :, 0], value_states[:, :, 0], o.pool.key_pool[l],
                            o.pool.value_pool[l], o._slots[:b])
        return key_states, value_states

    def get_seq_length(self) -> int:
        return 0

    def get_max_cache_shape(self) -> int:
        return self.owner.max_blocks * self.owner.bs

    def get_mask_sizes(self, query_length: int, *args, **kwargs):
        return self.owner.max_blocks * self.owner.bs, 0

    def lazy_initialization(self, *a, **k):
        pass

    def reset(self) -> None:
        pass


class GraphedPagedDecoder:
    """Decode one token for each of B sequences against the paged pool, as a graph."""

    def __init__(self, model, pool, max_batch: int, max_model_len: int, ctx_bucket: int = 32,
                 attn_kernel: str = "sm100", num_splits: int = 8):
        if attn_kernel != "sm100":
            raise ValueError(f"attn_kernel must be 'sm100' in this build, got {attn_kernel!r}")
        if not AB.register():
            raise RuntimeError("graphed paged decode needs the transformers attention registry")
        self.model, self.pool = model, pool
        self.device = torch.device(pool.key_pool.device)
        if self.device.type != "cuda":
            raise ValueError("graphed paged decode needs a CUDA device")
        self.bs = pool.block_size
        self.max_batch = max(1, max_batch)
        self.max_blocks = (max_model_len + 1 + self.bs - 1) // self.bs
        mb, dev = self.max_batch, self.device
        self._tok = torch.zeros((mb, 1), dtype=torch.long, device=dev)
        self._pos = torch.zeros(mb, dtype=torch.long, device=dev)
        self._table = torch.zeros((mb, self.max_blocks), dtype=torch.int32, device=dev)
        self._ctx = torch.ones(mb, dtype=torch.int32, device=dev)
        self._slots = torch.zeros(mb, dtype=torch.int32, device=dev)
        self.cache = Cache(layers=[_GraphLayer(self, i) for i in range(pool.spec.num_layers)])
        self._mem_pool = torch.cuda.graph_pool_handle()
        self._graphs: Dict[int, torch.cuda.CUDAGraph] = {}
        self._outs: Dict[int, torch.Tensor] = {}
        self._b = 1
        self.replays = 0
        self.captures = 0

    @staticmethod
    def _batch_bucket(b: int) -> int:
        p = 1
        while p < b:
            p *= 2
        return p

    @contextmanager
    def _bound(self, b: int):
        with AB.backend_enabled_on(self.model):
            with AB.graph_attention_context(self.pool, self._table[:b], self._ctx[:b]):
                yield

    @torch.no_grad()
    def _run(self, b: int):
        self._b = b
        bs = self.bs
        pos = self._pos[:b]
        rows = torch.arange(b, device=self.device)
        self._slots[:b].copy_(self._table[rows, pos // bs].long() * bs + pos % bs)
        self._ctx[:b].copy_(pos + 1)
        with self._bound(b):
            return self.model(input_ids=self._tok[:b], position_ids=pos[:, None],
                              past_key_values=self.cache, use_cache=True).logits[:, -1]

    @torch.no_grad()
    def _capture(self, b: int) -> None:
        stream = torch.cuda.Stream(self.device)
        stream.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(stream):
            for _ in range(2):
                self._run(b)
        torch.cuda.current_stream(self.device).wait_stream(stream)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, pool=self._mem_pool):
            out = self._run(b)
        self._graphs[b] = g
        self._outs[b] = out
        self.captures += 1

    @torch.no_grad()
    def step(self, tokens: Sequence[int], ctx_lens: Sequence[int],
             block_tables: Sequence[torch.Tensor]) -> torch.Tensor:
        """
        Decode one token per row.  ``ctx_lens[i]`` tokens are already cached for
        row i; the new token is written at that position (its block must be
        allocated).  Returns fresh logits ``(n, vocab)``.
        """
        n = len(tokens)
        if n == 0:
            raise ValueError("step() needs at least one sequence")
        b = self._batch_bucket(n)
        if b > self.max_batch:
            raise ValueError(f"batch {n} exceeds max_batch {self.max_batch}")
        if max(ctx_lens) + 1 > self.max_blocks * self.bs:
            raise ValueError(f"context {max(ctx_lens) + 1} exceeds the table width")
        for i, (c, t) in enumerate(zip(ctx_lens, block_tables)):
            if c // self.bs >= min(t.numel(), self.max_blocks):
                raise IndexError(f"row {i}: position {c} needs block {c // self.bs} but its "
                                 f"table has {t.numel()} entries")
        toks = list(tokens) + [tokens[0]] * (b - n)
        poss = list(ctx_lens) + [ctx_lens[0]] * (b - n)
        tabs = list(block_tables) + [block_tables[0]] * (b - n)
        self._tok[:b, 0].copy_(torch.tensor(toks, dtype=torch.long), non_blocking=False)
        self._pos[:b].copy_(torch.tensor(poss, dtype=torch.long), non_blocking=False)
        self._table[:b].zero_()
        for i, t in enumerate(tabs):
            t = t[: self.max_blocks]
            self._table[i, : t.numel()] = t.to(device=self.device, dtype=torch.int32)
        if b not in self._graphs:
            self._capture(b)
        self._graphs[b].replay()
        self.replays += 1
        return self._outs[b][:n].clone()
