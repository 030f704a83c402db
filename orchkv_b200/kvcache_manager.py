"""KVCacheManager on the B200 path.

Same constructor, public methods, statistics and decisions as the
reference's python/orchkv/kvcache_manager.py:43-566 (KVBlock, KVCacheManager):
blocks of `block_size` tokens per layer, each with its own [2, kv_heads,
block_size, head_dim] tensor on the GPU, in pinned DRAM or in a file
`<ssd_dir>/blk_<id>.bin`; eviction of the least-accessed GPU blocks above
85% of the GPU budget, spills of the least-accessed DRAM blocks when an SSD
directory is set, promotion of the most-accessed DRAM blocks below 60%.

What changes is where the per-block work of a decode step runs:

* ``report_attention``: the reference takes the mean over batch and query
  positions with torch, then for every block one ``float()`` device sync and
  one ``tm_report_attn`` call (:317-347).  Here the same mean feeds one
  ``tm_report_attn_ranges`` launch that sums every block's token range over
  all heads and records it in the tracker; the access counts are bumped on
  the host for the blocks it reports.
* ``build_past_kv`` concatenates each layer's block slices with one
  ``torch.cat`` per tensor instead of one copy per block (:270-315); the
  result is the same.

Block ids come from a counter, registered with the reference binding's
positional quirk (``tm_register_block_id(tm, bid, flags, GPU_HBM)``: a sink
block lands on tier 1, :157-161).  Blocks whose ids would share a tracker
slot with another block of the same report are reported one by one, in
block order, as the reference does.
"""
from __future__ import annotations

import logging
import os
from dataclasses import dataclass
from pathlib import Path
from typing import Optional

import numpy as np
import torch

from . import core

try:
    from transformers import DynamicCache
    HAS_DYNAMIC_CACHE = True
except ImportError:  # pragma: no cover - transformers is part of the image
    HAS_DYNAMIC_CACHE = False

logger = logging.getLogger(__name__)

TIER_GPU = 0
TIER_DRAM = 1
TIER_SSD = 2

_TIER_NAMES = {TIER_GPU: "GPU", TIER_DRAM: "DRAM", TIER_SSD: "SSD"}


@dataclass
class KVBlock:
    """One block of one layer's KV cache and where its data lives."""
    block_id: int
    layer: int
    token_start: int
    token_count: int = 0
    capacity: int = 16
    tier: int = TIER_GPU
    gpu_data: Optional[torch.Tensor] = None
    dram_data: Optional[torch.Tensor] = None
    ssd_path: Optional[str] = None
    is_sink: bool = False
    access_count: int = 0


class KVCacheManager:
    """Block-level KV-cache manager over GPU, DRAM and SSD tiers."""

    def __init__(self, n_layers: int, n_kv_heads: int, head_dim: int, block_size: int = 16,
                 dtype: torch.dtype = torch.float16, gpu_budget_bytes: int = 0,
                 ssd_dir: Optional[str] = None, sink_tokens: int = 4):
        self.n_layers = n_layers
        self.n_kv_heads = n_kv_heads
        self.head_dim = head_dim
        self.block_size = block_size
        self.dtype = dtype
        self.gpu_budget_bytes = gpu_budget_bytes
        self.ssd_dir = ssd_dir
        self.sink_tokens = sink_tokens
        self._block_bytes = 2 * n_kv_heads * block_size * head_dim * dtype.itemsize
        self._next_block_id = 0
        self._total_tokens = 0
        self._blocks: list[list[KVBlock]] = [[] for _ in range(n_layers)]
        self._step = 0
        self._stats = {"gpu_to_dram": 0, "dram_to_gpu": 0, "dram_to_ssd": 0,
                       "ssd_to_dram": 0, "total_blocks": 0}
        if ssd_dir:
            Path(ssd_dir).mkdir(parents=True, exist_ok=True)
        self._C = core()
        self._tm_handle: Optional[int] = self._C.tm_create()
        self._cap = int(self._C.tm_capacity(self._tm_handle))
        self._tm_stream = None

    def destroy(self):
        if self._tm_handle is not None:
            self._C.tm_destroy(self._tm_handle)
            self._tm_handle = None

    # -- sizes ------------------------------------------------------------------
    @property
    def total_tokens(self) -> int:
        return self._total_tokens

    @property
    def block_bytes(self) -> int:
        return self._block_bytes

    def _all_blocks(self):
        for layer_blocks in self._blocks:
            yield from layer_blocks

    def gpu_kv_bytes(self) -> int:
        return sum(1 for b in self._all_blocks() if b.tier == TIER_GPU) * self._block_bytes

    # -- blocks -------------------------------------------------------------------
    def _alloc_block(self, layer: int, token_start: int) -> KVBlock:
        bid = self._next_block_id
        self._next_block_id += 1
        sink = token_start < self.sink_tokens
        blk = KVBlock(block_id=bid, layer=layer, token_start=token_start,
                      capacity=self.block_size, is_sink=sink)
        self._blocks[layer].append(blk)
        self._stats["total_blocks"] += 1
        if self._tm_handle is not None:
            # positional, as the reference calls it: tier := flags, flags := GPU_HBM
            self._C.tm_register_block_id(self._tm_handle, bid, 1 if sink else 0,
                                         int(self._C.GPU_HBM))
        return blk

    def _make_block_tensor(self, device: str = "cuda") -> torch.Tensor:
        shape = (2, self.n_kv_heads, self.block_size, self.head_dim)
        if device == "cpu":
            return torch.zeros(*shape, dtype=self.dtype, device="cpu", pin_memory=True)
        return torch.zeros(*shape, dtype=self.dtype, device="cuda")

    # -- past_key_values formats ------------------------------------------------------
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
            return DynamicCache(ddp_cache_data=legacy_cache)
        return legacy_cache

    # -- ingest -------------------------------------------------------------------------
    def ingest_step(self, past_key_values) -> None:
        """Take in the KV cache of a forward pass (positions not yet managed)."""
        legacy = self._to_legacy(past_key_values)
        for layer, (k, v) in enumerate(legacy):
            self._ingest_layer(layer, k, v, k.shape[2])
        self._total_tokens = legacy[0][0].shape[2]

    def _ingest_layer(self, layer: int, key: torch.Tensor, value: torch.Tensor, seq_len: int):
        have = sum(b.token_count for b in self._blocks[layer])
        for pos in range(have, seq_len, self.block_size):
            end = min(pos + self.block_size, seq_len)
            blk = self._alloc_block(layer, pos)
            blk.token_count = end - pos
            data = self._make_block_tensor("cuda")
            data[0, :, :end - pos] = key[0, :, pos:end]
            data[1, :, :end - pos] = value[0, :, pos:end]
            blk.gpu_data = data
            blk.tier = TIER_GPU

    def append_token(self, past_key_values) -> None:
        """Take in only the newest position of every layer."""
        legacy = self._to_legacy(past_key_values)
        for layer, (k, v) in enumerate(legacy):
            seq_len = k.shape[2]
            blocks = self._blocks[layer]
            if not blocks:
                self._ingest_layer(layer, k, v, seq_len)
                continue
            have = sum(b.token_count for b in blocks)
            if seq_len <= have:
                continue
            last = blocks[-1]
            if last.token_count < last.capacity:
                if last.tier != TIER_GPU:
                    self._promote_block(last)
                last.gpu_data[0, :, last.token_count] = k[0, :, -1]
                last.gpu_data[1, :, last.token_count] = v[0, :, -1]
                last.token_count += 1
            else:
                blk = self._alloc_block(layer, have)
                blk.token_count = 1
                data = self._make_block_tensor("cuda")
                data[0, :, 0] = k[0, :, -1]
                data[1, :, 0] = v[0, :, -1]
                blk.gpu_data = data
        self._total_tokens = legacy[0][0].shape[2]

    # -- build -------------------------------------------------------------------------
    def build_past_kv(self, device: str = "cuda"):
        """past_key_values of every managed position, promoting blocks that are
        not on the GPU first."""
        out = []
        for layer in range(self.n_layers):
            blocks = [b for b in self._blocks[layer] if b.token_count > 0]
            if not blocks:
                empty = torch.zeros(1, self.n_kv_heads, 0, self.head_dim, dtype=self.dtype,
                                    device=device)
                out.append((empty, empty.clone()))
                continue
            for b in blocks:
                if b.tier != TIER_GPU:
                    self._promote_block(b)
            key = torch.cat([b.gpu_data[0, :, :b.token_count] for b in blocks], dim=1)
            val = torch.cat([b.gpu_data[1, :, :b.token_count] for b in blocks], dim=1)
            out.append((key.unsqueeze(0).to(device), val.unsqueeze(0).to(device)))
        return self._from_legacy(tuple(out))

    # -- attention reports ------------------------------------------------------------------
    def _bind_stream(self):
        s = torch.cuda.current_stream().cuda_stream
        if s != self._tm_stream:
            self._C.tm_set_stream(self._tm_handle, s)
            self._tm_stream = s

    def report_attention(self, layer_idx: int, attn_weights: torch.Tensor):
        """Per-block attention mass of one layer: the sum over heads and the
        block's tokens of the weights averaged over batch and query positions."""
        if self._tm_handle is None:
            return
        blocks = self._blocks[layer_idx]
        if not blocks:
            return
        with torch.no_grad():
            avg = attn_weights.float().mean(dim=(0, 2)).contiguous()   # [heads, kv_len]
            heads, kv_len = avg.shape
            starts = np.fromiter((b.token_start for b in blocks), np.int64, len(blocks))
            ends = np.minimum(starts + np.fromiter((b.token_count for b in blocks), np.int64,
                                                   len(blocks)), kv_len)
            live = starts < ends
            if not live.any():
                return
            ids = np.fromiter((b.block_id for b in blocks), np.int64, len(blocks))[live]
            slots = ids & (self._cap - 1)
            if len(np.unique(slots)) == len(slots) and ids.max() < 0xFFFFFFFF:
                self._bind_stream()
                arr = np.stack([starts[live], ends[live], ids]).astype(np.uint32)
                rc = self._C.tm_report_attn_ranges(self._tm_handle, avg.data_ptr(), heads,
                                                   kv_len, arr[0].ctypes.data,
                                                   arr[1].ctypes.data, arr[2].ctypes.data,
                                                   len(ids))
                if rc != 0:
                    raise RuntimeError(f"tm_report_attn_ranges failed: {rc}")
            else:
                # two blocks on one tracker slot: one report per block, in order
                for s, e, bid in zip(starts[live], ends[live], ids):
                    self._C.tm_report_attn(self._tm_handle, int(bid),
                                           float(avg[:, int(s):int(e)].sum()))
            for b, reported in zip(blocks, live):
                if reported:
                    b.access_count += 1

    # -- scheduling ---------------------------------------------------------------------------
    def step_done(self):
        self._step += 1
        if self._tm_handle is not None:
            self._bind_stream()
            self._C.tm_step_done(self._tm_handle)

    def schedule(self) -> dict:
        """One cycle: usage to the manager, its schedule pass, then the
        manager-side evictions, spills and promotions."""
        if self._tm_handle is None:
            return {}
        gpu_bytes = self.gpu_kv_bytes()
        budget = self.gpu_budget_bytes
        ratio = min(gpu_bytes / budget, 1.0) if budget > 0 else 0.0
        self._bind_stream()
        self._C.tm_set_usage(self._tm_handle, ratio, 0.0)
        self._C.tm_schedule_once(self._tm_handle)
        raw = self._C.tm_get_stats(self._tm_handle)
        evicted = promoted = 0
        if budget > 0 and gpu_bytes > budget * 0.85:
            evicted = self._evict_cold_blocks()
        if self.ssd_dir:
            self._spill_dram_to_ssd()
        if budget > 0 and gpu_bytes < budget * 0.60:
            promoted = self._promote_warm_blocks()
        return {"step": self._step, "gpu_kv_bytes": gpu_bytes, "gpu_ratio": ratio,
                "evicted": evicted, "promoted": promoted, "tm_stats": raw}

    def _evict_cold_blocks(self, max_evict: int = 8) -> int:
        """Least-accessed non-sink GPU blocks to DRAM until 70% of the budget."""
        cands = [b for b in self._all_blocks()
                 if b.tier == TIER_GPU and not b.is_sink and b.gpu_data is not None]
        cands.sort(key=lambda b: b.access_count)                 # stable: block order on ties
        evicted = 0
        for b in cands[:max_evict]:
            if self.gpu_budget_bytes > 0 and self.gpu_kv_bytes() <= self.gpu_budget_bytes * 0.7:
                break
            self._demote_block(b)
            evicted += 1
        return evicted

    def _promote_warm_blocks(self, max_promote: int = 4) -> int:
        """Most-accessed DRAM blocks back to the GPU."""
        cands = [b for b in self._all_blocks() if b.tier == TIER_DRAM and b.dram_data is not None]
        cands.sort(key=lambda b: b.access_count, reverse=True)
        for b in cands[:max_promote]:
            self._promote_block(b)
        return min(len(cands), max_promote)

    def _spill_dram_to_ssd(self, max_spill: int = 4):
        """Least-accessed non-sink DRAM blocks to files, once at least 4 are in DRAM."""
        dram = [b for b in self._all_blocks()
                if b.tier == TIER_DRAM and b.dram_data is not None and not b.is_sink]
        if len(dram) < 4:
            return
        dram.sort(key=lambda b: b.access_count)
        for b in dram[:max_spill]:
            self._save_to_ssd(b)

    # -- data movement ---------------------------------------------------------------------
    def _demote_block(self, blk: KVBlock):
        if blk.tier != TIER_GPU or blk.gpu_data is None:
            return
        if blk.dram_data is None:
            blk.dram_data = torch.empty_like(blk.gpu_data, device="cpu", pin_memory=True)
        blk.dram_data.copy_(blk.gpu_data)
        blk.gpu_data = None
        blk.tier = TIER_DRAM
        self._stats["gpu_to_dram"] += 1
        if self._tm_handle is not None:
            self._C.tm_set_block_tier(self._tm_handle, blk.block_id, int(self._C.HOST_DRAM))

    def _promote_block(self, blk: KVBlock):
        if blk.tier == TIER_SSD:
            self._load_from_ssd(blk)
        if blk.tier == TIER_DRAM and blk.dram_data is not None:
            blk.gpu_data = blk.dram_data.to("cuda")
            blk.tier = TIER_GPU
            self._stats["dram_to_gpu"] += 1
            if self._tm_handle is not None:
                self._C.tm_set_block_tier(self._tm_handle, blk.block_id, int(self._C.GPU_HBM))

    def _save_to_ssd(self, blk: KVBlock):
        if self.ssd_dir is None or blk.dram_data is None:
            return
        path = os.path.join(self.ssd_dir, f"blk_{blk.block_id}.bin")
        with open(path, "wb") as fh:                  # the tensor's raw bytes (any dtype)
            fh.write(blk.dram_data.contiguous().view(torch.uint8).numpy().tobytes())
        blk.ssd_path = path
        blk.dram_data = None
        blk.tier = TIER_SSD
        self._stats["dram_to_ssd"] += 1
        if self._tm_handle is not None:
            self._C.tm_set_block_tier(self._tm_handle, blk.block_id, int(self._C.SSD))

    def _load_from_ssd(self, blk: KVBlock):
        if blk.ssd_path is None or not os.path.exists(blk.ssd_path):
            return
        with open(blk.ssd_path, "rb") as fh:
            raw = bytearray(fh.read())
        shape = (2, self.n_kv_heads, self.block_size, self.head_dim)
        data = torch.frombuffer(raw, dtype=torch.uint8).view(self.dtype).reshape(shape)
        blk.dram_data = data.clone().pin_memory()
        blk.tier = TIER_DRAM
        self._stats["ssd_to_dram"] += 1

    # -- statistics -----------------------------------------------------------------------
    def get_stats(self) -> dict:
        n = {TIER_GPU: 0, TIER_DRAM: 0, TIER_SSD: 0}
        for b in self._all_blocks():
            if b.tier in n:
                n[b.tier] += 1
        tm_stats = self._C.tm_get_stats(self._tm_handle) if self._tm_handle is not None else {}
        return {"step": self._step, "total_tokens": self._total_tokens,
                "blocks_gpu": n[TIER_GPU], "blocks_dram": n[TIER_DRAM], "blocks_ssd": n[TIER_SSD],
                "blocks_total": sum(n.values()),
                "gpu_kv_mb": n[TIER_GPU] * self._block_bytes / (1 << 20),
                "dram_kv_mb": n[TIER_DRAM] * self._block_bytes / (1 << 20),
                "migrations": dict(self._stats), "tm": tm_stats}

    def __repr__(self) -> str:
        s = self.get_stats()
        return (f"KVCacheManager(tokens={s['total_tokens']}, blocks={s['blocks_total']} "
                f"[GPU:{s['blocks_gpu']} DRAM:{s['blocks_dram']} SSD:{s['blocks_ssd']}], "
                f"gpu_kv={s['gpu_kv_mb']:.1f}MB)")
