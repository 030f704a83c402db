"""FastKVCacheManager on the B200 path.

Same constructor, public methods, buffers, statistics and decisions as the
reference's python/orchkv/fast_kvcache_manager.py:44-365, so an HF decode
loop written against it switches by import.  The per-block Python work of
the decode step is replaced by single launches:

* ``report_attention`` / ``report_qk_norm``: one ``tm_report_attn_probs``
  launch per layer reduces the whole [q-heads, tokens] map to per-block
  mass and records it (the reference: one ``float()`` device sync and one
  ``tm_report_attn`` call per block, :221-270);
* cold-block eviction: one ``tm_select_victims_masked`` selection (coldest
  by hotness, ties by block id, the reference's stable sort over
  ``tm_get_block_score``, :300-321) and one ``orchkv_copy_token_blocks``
  launch moving the chosen blocks of every layer into a pinned store (the
  reference: a ``.cpu()`` per block and layer, :324-338);
* the restore in ``build_past_kv``: one launch per eviction batch (the
  reference: a ``.to("cuda")`` per range and layer, :204-219).

Block ids are token-block indices shared by all layers, registered with the
reference binding's positional quirk (``tm_register_block_id(tm, bid,
flags, 0)``: sink blocks land on tier 1), as the reference does (:155,173).
The reference's unused ``_block_scores`` side table is not kept.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path
from typing import Optional

import torch

from . import core, lib
from ._lib import TieredManager

try:
    from transformers import DynamicCache
    HAS_DYNAMIC_CACHE = True
except ImportError:  # pragma: no cover - transformers is part of the image
    HAS_DYNAMIC_CACHE = False

TIER_GPU = 0
TIER_DRAM = 1
TIER_SSD = 2


class _DeviceKV:
    """Every layer's persistent K and V in one device tensor
    [2 (K, V), layers, 1, kv heads, capacity tokens, head_dim].  Per-layer
    views keep the [1, heads, tokens, head_dim] shape of a legacy cache
    entry, and the K/V pointers of all layers are what one
    orchkv_copy_token_blocks launch gathers from or scatters into."""

    def __init__(self, layers: int, heads: int, head_dim: int, dtype: torch.dtype,
                 capacity: int):
        self.layers, self.heads, self.head_dim, self.dtype = layers, heads, head_dim, dtype
        self.t = torch.zeros(2, layers, 1, heads, capacity, head_dim, dtype=dtype, device="cuda")

    @property
    def capacity(self) -> int:
        return self.t.shape[4]

    def layer(self, li: int) -> tuple[torch.Tensor, torch.Tensor]:
        return self.t[0, li], self.t[1, li]

    def store(self, li: int, pos: int, k: torch.Tensor, v: torch.Tensor) -> None:
        """Write k, v [heads, n, head_dim] at token positions [pos, pos + n)."""
        n = k.shape[1]
        self.t[0, li, 0, :, pos:pos + n] = k
        self.t[1, li, 0, :, pos:pos + n] = v

    def grow(self, capacity: int) -> None:
        """Reallocate for `capacity` tokens, keeping the tokens that fit."""
        new = torch.zeros(2, self.layers, 1, self.heads, capacity, self.head_dim,
                          dtype=self.dtype, device="cuda")
        keep = min(capacity, self.capacity)
        new[..., :keep, :] = self.t[..., :keep, :]
        self.t = new

    def pointers(self) -> list[int]:
        """K then V of layer 0, K then V of layer 1, ..."""
        return [self.t[kv, li].data_ptr() for li in range(self.layers) for kv in (0, 1)]

    def head_stride_bytes(self) -> int:
        return self.t.stride(3) * self.t.element_size()


class FastKVCacheManager:
    """KV-cache manager with persistent per-layer buffers; scoring,
    selection and block movement run as single GPU launches."""

    def __init__(self, n_layers: int, n_kv_heads: int, head_dim: int, block_size: int = 16,
                 dtype: torch.dtype = torch.float16, gpu_budget_bytes: int = 0,
                 max_seq_len: int = 4096, ssd_dir: Optional[str] = None,
                 sink_tokens: int = 4):
        # the reference's public attributes (fast_kvcache_manager.py:44-60)
        self.n_layers, self.n_kv_heads, self.head_dim = n_layers, n_kv_heads, head_dim
        self.block_size, self.dtype = block_size, dtype
        self.gpu_budget_bytes, self.max_seq_len = gpu_budget_bytes, max_seq_len
        self.ssd_dir, self.sink_tokens = ssd_dir, sink_tokens
        self._row_bytes = head_dim * dtype.itemsize
        if self._row_bytes % 16:
            raise ValueError("head_dim * itemsize must be a multiple of 16 bytes")
        self._block_bytes = 2 * n_kv_heads * block_size * self._row_bytes
        self._kv = _DeviceKV(n_layers, n_kv_heads, head_dim, dtype, max_seq_len)
        self._total_tokens = 0
        self._step = 0
        # evicted block -> (start, end) token range at eviction; batches of
        # (first store slot, device block list, count, tokens at eviction)
        self._evicted: dict[int, tuple[int, int]] = {}
        self._batches: list[tuple[int, torch.Tensor, int, int]] = []
        self._store: Optional[torch.Tensor] = None
        self._store_used = 0
        self._stats = dict.fromkeys(("gpu_to_dram", "dram_to_gpu", "dram_to_ssd", "ssd_to_dram",
                                     "total_blocks", "evictions_this_step"), 0)

        self._C = core()
        self._tm_handle: Optional[int] = self._C.tm_create()
        self._tm_stream = None
        self._cap = lib().tm_capacity(self.tm_ref())
        self._ids = torch.arange(max(self._cap, max_seq_len // block_size + 1),
                                 dtype=torch.int32, device="cuda")
        self._lens = torch.zeros(1, dtype=torch.int32, device="cuda")
        self._mask = torch.zeros(self._cap, dtype=torch.uint8, device="cuda")
        self._sel = torch.zeros(64, dtype=torch.int32, device="cuda")
        self._cnt = torch.zeros(1, dtype=torch.int32, device="cuda")
        if ssd_dir:
            Path(ssd_dir).mkdir(parents=True, exist_ok=True)

    # -- lifecycle ---------------------------------------------------------

    def tm_ref(self):
        """The manager's tiered_manager_t for the C ABI (orchkv_b200.lib())."""
        return C.cast(C.c_void_p(self._tm_handle), C.POINTER(TieredManager))

    def destroy(self):
        if self._tm_handle is not None:
            self._C.tm_destroy(self._tm_handle)
            self._tm_handle = None

    @property
    def total_tokens(self) -> int:
        return self._total_tokens

    @property
    def _key_bufs(self) -> list[torch.Tensor]:
        return [self._kv.layer(li)[0] for li in range(self.n_layers)]

    @property
    def _val_bufs(self) -> list[torch.Tensor]:
        return [self._kv.layer(li)[1] for li in range(self.n_layers)]

    @property
    def _evicted_ranges(self) -> list[list[tuple[int, int]]]:
        """Per layer, the evicted token ranges (the reference's bookkeeping)."""
        r = sorted(self._evicted.values())
        return [list(r) for _ in range(self.n_layers)]

    def _n_blocks(self) -> int:
        return (self._total_tokens + self.block_size - 1) // self.block_size

    def gpu_kv_bytes(self) -> int:
        return (self._n_blocks() - len(self._evicted)) * self.n_layers * self._block_bytes

    def _stream(self) -> int:
        return torch.cuda.current_stream().cuda_stream

    def _sync_tm_stream(self):
        """Run the manager's GPU work on torch's current stream (rebinding
        synchronises the old stream, so only when it changed)."""
        s = self._stream()
        if s != self._tm_stream:
            self._C.tm_set_stream(self._tm_handle, s)
            self._tm_stream = s

    # -- ingest ------------------------------------------------------------

    @staticmethod
    def _to_legacy(past_key_values):
        if HAS_DYNAMIC_CACHE and isinstance(past_key_values, DynamicCache):
            if hasattr(past_key_values, "to_legacy_cache"):
                return past_key_values.to_legacy_cache()
            return tuple((lay.keys, lay.values) for lay in past_key_values.layers)
        return past_key_values

    @staticmethod
    def _from_legacy(legacy_cache):
        if HAS_DYNAMIC_CACHE:
            if hasattr(DynamicCache, "from_legacy_cache"):
                return DynamicCache.from_legacy_cache(legacy_cache)
            return DynamicCache(ddp_cache_data=legacy_cache)    # transformers >= 5
        return legacy_cache

    def _register(self, first_block: int, last_block: int) -> None:
        """Register token blocks [first, last) with the scheduler.  Blocks
        holding sink tokens carry flag 1, passed in the binding's tier
        position as the reference does (fast_kvcache_manager.py:155,173:
        tm_register_block_id(tm, bid, flags, 0))."""
        for bid in range(first_block, last_block):
            sink = 1 if bid * self.block_size < self.sink_tokens else 0
            self._C.tm_register_block_id(self._tm_handle, bid, sink, 0)

    def _ensure_capacity(self, tokens: int) -> None:
        """Buffers for at least `tokens` tokens, grown in steps of 256."""
        if tokens <= self._kv.capacity:
            return
        self._grow_buffers(tokens)

    def _grow_buffers(self, new_max: int):
        new_max = -(-new_max // 256) * 256
        self._kv.grow(new_max)
        self.max_seq_len = new_max
        need = new_max // self.block_size + 1
        if self._ids.numel() < need:
            self._ids = torch.arange(need, dtype=torch.int32, device="cuda")

    def ingest_step(self, past_key_values) -> None:
        """Take a prefill's cache: every layer's tokens into the buffers and
        every token block registered."""
        layers = self._to_legacy(past_key_values)
        for li, (k, v) in enumerate(layers):
            n = k.shape[2]
            self._ensure_capacity(n)
            self._kv.store(li, 0, k[0, :, :n], v[0, :, :n])
        self._total_tokens = layers[0][0].shape[2]
        n_blocks = self._n_blocks()
        self._register(0, n_blocks)
        self._stats["total_blocks"] = n_blocks * self.n_layers

    def append_token(self, past_key_values) -> None:
        """Take one decode step's token (the last position of each layer's
        cache); a token that opens a block registers the block."""
        layers = self._to_legacy(past_key_values)
        pos = self._total_tokens
        if pos >= self._kv.capacity:
            self._grow_buffers(pos + 256)
        for li, (k, v) in enumerate(layers):
            self._kv.store(li, pos, k[0, :, -1:], v[0, :, -1:])
        self._total_tokens = pos + 1
        if pos % self.block_size == 0:
            self._register(pos // self.block_size, pos // self.block_size + 1)

    # -- block movement ----------------------------------------------------

    def _slot_elems(self) -> int:
        return 2 * self.n_layers * self.n_kv_heads * self.block_size * self.head_dim

    def _reserve_store(self, n: int) -> int:
        """First store slot of n new blocks (grows the pinned store)."""
        need = self._store_used + n
        if self._store is None or self._store.shape[0] < need:
            cap = max(need, 2 * (0 if self._store is None else self._store.shape[0]), 16)
            new = torch.empty(cap, self._slot_elems(), dtype=self.dtype).pin_memory()
            if self._store is not None and self._store_used:
                torch.cuda.current_stream().synchronize()
                new[: self._store_used].copy_(self._store[: self._store_used])
            self._store = new
        first = self._store_used
        self._store_used = need
        return first

    def _copy_blocks(self, blocks: torch.Tensor, n: int, n_tokens: int, slot: int, direction: int):
        store_ptr = self._store.data_ptr() + slot * self._slot_elems() * self.dtype.itemsize
        rc = self._C.copy_token_blocks(self._kv.pointers(), self.n_kv_heads,
                                       self._kv.head_stride_bytes(),
                                       self._row_bytes, self.block_size, n_tokens,
                                       blocks.data_ptr(), n, store_ptr, direction, self._stream())
        if rc != 0:
            raise RuntimeError(f"orchkv_copy_token_blocks failed: {rc}")

    # -- build -------------------------------------------------------------

    def build_past_kv(self, device: str = "cuda"):
        n = self._total_tokens
        self._restore_evicted_blocks()
        return self._from_legacy(tuple((k[:, :, :n], v[:, :, :n])
                                       for k, v in map(self._kv.layer, range(self.n_layers))))

    def _restore_evicted_blocks(self):
        for slot, blocks, n, n_tokens in self._batches:
            self._copy_blocks(blocks, n, n_tokens, slot, 1)
            self._stats["dram_to_gpu"] += n * self.n_layers
        self._batches.clear()
        self._evicted.clear()
        self._store_used = 0

    # -- attention reporting -----------------------------------------------

    def _report_map(self, m: torch.Tensor, n_tokens: int):
        """m: [heads, T] float32; every head's mass of each block -> block id."""
        m = m.contiguous()
        n_tok = min(n_tokens, m.shape[-1])
        if n_tok <= 0:
            return
        self._lens.fill_(n_tok)
        self._sync_tm_stream()
        rc = self._C.tm_report_attn_probs(self._tm_handle, m.data_ptr(), 1, m.shape[0], 1,
                                          m.shape[-1], self.block_size, self._ids.data_ptr(),
                                          self._lens.data_ptr())
        if rc != 0:
            raise RuntimeError(f"tm_report_attn_probs failed: {rc}")

    def report_attention(self, layer_idx: int, attn_weights: torch.Tensor):
        if self._tm_handle is None:
            return
        with torch.no_grad():
            avg = attn_weights.float().mean(dim=(0, 2))            # [q-heads, T]
            self._report_map(avg, self._total_tokens)

    def report_qk_norm(self, layer_idx: int, q: torch.Tensor):
        """QK-norm proxy (fast_kvcache_manager.py:237-270): |q . K| per token,
        summed over heads and block tokens."""
        if self._tm_handle is None:
            return
        n = self._total_tokens
        if n == 0:
            return
        with torch.no_grad():
            gqa_ratio = q.shape[1] // self.n_kv_heads
            q_for_kv = q[:, ::gqa_ratio, :, :] if gqa_ratio > 1 else q
            k_all = self._kv.layer(layer_idx)[0][:, :, :n, :]
            qk = torch.matmul(q_for_kv, k_all.transpose(-1, -2))
            qk_abs = qk.abs().squeeze(0).squeeze(1).float()
            self._report_map(qk_abs, n)

    # -- scheduling --------------------------------------------------------

    def step_done(self):
        self._step += 1
        if self._tm_handle is not None:
            self._sync_tm_stream()
            self._C.tm_step_done(self._tm_handle)

    def schedule(self) -> dict:
        if self._tm_handle is None:
            return {}
        n_blocks = self._n_blocks()
        evicted_count = len(self._evicted) * self.n_layers
        total_block_layers = n_blocks * self.n_layers
        gpu_ratio = 1.0 - evicted_count / total_block_layers if total_block_layers > 0 else 0.0
        self._sync_tm_stream()
        self._C.tm_set_usage(self._tm_handle, gpu_ratio, 0.0)
        self._C.tm_schedule_once(self._tm_handle)
        self._stats["evictions_this_step"] = 0
        if self.gpu_budget_bytes > 0 and self.gpu_kv_bytes() > self.gpu_budget_bytes * 0.85:
            self._evict_cold_blocks()
        return {"step": self._step, "gpu_ratio": gpu_ratio}

    def _evict_cold_blocks(self, max_evict: int = 8) -> int:
        n_blocks = self._n_blocks()
        first = min((self.sink_tokens + self.block_size - 1) // self.block_size, n_blocks)
        n_cand = n_blocks - first - sum(1 for b in self._evicted if b >= first)
        if n_cand <= 0 or max_evict <= 0:
            return 0
        # the reference evicts coldest-first and stops once the GPU bytes are
        # at most 85% of the budget: that many blocks, at most max_evict
        per_block = self.n_layers * self._block_bytes
        k, gb = 1, self.gpu_kv_bytes() - per_block
        while k < min(max_evict, n_cand) and not gb <= self.gpu_budget_bytes * 0.85:
            k += 1
            gb -= per_block
        # candidates: blocks [first, n_blocks) not evicted (block id = slot)
        self._mask.zero_()
        self._mask[first:n_blocks] = 1
        if self._evicted:
            ev = torch.tensor(sorted(self._evicted), dtype=torch.long, device="cuda")
            self._mask[ev] = 0
        self._sync_tm_stream()
        rc = self._C.tm_select_victims_masked(self._tm_handle, k, self._mask.data_ptr(),
                                              self._sel.data_ptr(), self._cnt.data_ptr())
        if rc != 0:
            raise RuntimeError(f"tm_select_victims_masked failed: {rc}")
        c = int(self._cnt.item())
        if c == 0:
            return 0
        blocks = self._sel[:c].clone()
        slot = self._reserve_store(c)
        self._copy_blocks(blocks, c, self._total_tokens, slot, 0)
        for bid in blocks.tolist():
            start = bid * self.block_size
            self._evicted[bid] = (start, min(start + self.block_size, self._total_tokens))
        self._batches.append((slot, blocks, c, self._total_tokens))
        self._stats["gpu_to_dram"] += c * self.n_layers
        self._stats["evictions_this_step"] += c
        return c

    # -- stats -------------------------------------------------------------

    def get_stats(self) -> dict:
        """The reference's statistics dict (fast_kvcache_manager.py:347-360):
        block counts over all layers, the GPU-resident KV in MiB, and the
        migration counters."""
        total = self._n_blocks() * self.n_layers
        off_gpu = len(self._evicted) * self.n_layers
        on_gpu = total - off_gpu
        return {"step": self._step, "total_tokens": self._total_tokens,
                "blocks_gpu": on_gpu, "blocks_dram": off_gpu, "blocks_ssd": 0,
                "blocks_total": total, "gpu_kv_mb": on_gpu * self._block_bytes / (1 << 20),
                "migrations": dict(self._stats)}

    def __repr__(self) -> str:
        on_gpu = (self._n_blocks() - len(self._evicted)) * self.n_layers
        return (f"FastKVCacheManager(tokens={self._total_tokens}, gpu={on_gpu}, "
                f"dram={len(self._evicted) * self.n_layers})")
