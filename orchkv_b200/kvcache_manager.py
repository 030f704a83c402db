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

The bookkeeping is organised around tier moves: every change of a block's
tier goes through ``_relocate``, which moves the bytes, counts the move
under the statistic the reference keeps for it and tells the tracker the
new tier where the reference does (not for a file read back into DRAM,
:513-527); eviction, spill and promotion candidates come from one stable
ranking by access count (``_ranked``).

Block ids come from a counter, registered with the reference binding's
positional quirk (``tm_register_block_id(tm, bid, flags, GPU_HBM)``: a sink
block lands on tier 1, :157-161).  Blocks whose ids would share a tracker
slot with another block of the same report are reported one by one, in
block order, as the reference does.
"""
from __future__ import annotations

import logging
import os
from collections import Counter
from dataclasses import dataclass
from operator import attrgetter
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

# the statistic each tier move counts under, in the order get_stats lists them
_MOVES = {(TIER_GPU, TIER_DRAM): "gpu_to_dram", (TIER_DRAM, TIER_GPU): "dram_to_gpu",
          (TIER_DRAM, TIER_SSD): "dram_to_ssd", (TIER_SSD, TIER_DRAM): "ssd_to_dram"}

# GPU-budget thresholds of one schedule cycle (kvcache_manager.py:381, 387, 422)
_EVICT_ABOVE, _EVICT_DOWN_TO, _PROMOTE_BELOW = 0.85, 0.70, 0.60


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
        self.n_layers, self.n_kv_heads, self.head_dim = n_layers, n_kv_heads, head_dim
        self.block_size, self.dtype = block_size, dtype
        self.gpu_budget_bytes, self.ssd_dir, self.sink_tokens = gpu_budget_bytes, ssd_dir, sink_tokens
        self._shape = (2, n_kv_heads, block_size, head_dim)      # one block: [K|V][head][token][d]
        self._block_bytes = int(np.prod(self._shape)) * dtype.itemsize
        self._blocks: list[list[KVBlock]] = [[] for _ in range(n_layers)]
        self._ids = 0                                            # next block id
        self._total_tokens = 0
        self._step = 0
        self._moves: Counter = Counter()
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

    def _every_block(self):
        """All blocks, layer by layer, each layer's in token order."""
        for layer in self._blocks:
            yield from layer

    def _tier_counts(self) -> Counter:
        return Counter(b.tier for b in self._every_block())

    def gpu_kv_bytes(self) -> int:
        return self._tier_counts()[TIER_GPU] * self._block_bytes

    # -- past_key_values formats ---------------------------------------------------
    @staticmethod
    def _to_legacy(past_key_values):
        """(key, value) per layer, from a DynamicCache or a legacy tuple."""
        if not (HAS_DYNAMIC_CACHE and isinstance(past_key_values, DynamicCache)):
            return past_key_values
        convert = getattr(past_key_values, "to_legacy_cache", None)
        if convert is not None:
            return convert()
        return tuple((lay.keys, lay.values) for lay in past_key_values.layers)

    @staticmethod
    def _from_legacy(legacy_cache):
        """The DynamicCache HF models take back (the tuple where there is none)."""
        if not HAS_DYNAMIC_CACHE:
            return legacy_cache
        build = getattr(DynamicCache, "from_legacy_cache", None)
        return build(legacy_cache) if build is not None else DynamicCache(ddp_cache_data=legacy_cache)

    # -- blocks -------------------------------------------------------------------
    def _new_block(self, layer: int, token_start: int) -> KVBlock:
        """A zeroed GPU block at the end of `layer`, registered with the tracker
        as the reference registers it (tier := sink flag, flags := GPU_HBM)."""
        blk = KVBlock(block_id=self._ids, layer=layer, token_start=token_start,
                      capacity=self.block_size, is_sink=token_start < self.sink_tokens,
                      gpu_data=torch.zeros(self._shape, dtype=self.dtype, device="cuda"))
        self._ids += 1
        self._blocks[layer].append(blk)
        if self._tm_handle is not None:
            self._C.tm_register_block_id(self._tm_handle, blk.block_id, int(blk.is_sink),
                                         int(self._C.GPU_HBM))
        return blk

    def _held(self, layer: int) -> int:
        return sum(b.token_count for b in self._blocks[layer])

    def _absorb_range(self, layer: int, key: torch.Tensor, value: torch.Tensor, upto: int):
        """New blocks for positions [held, upto) of `layer`, block_size at a time
        (a partly filled last block is left as it is, as the reference does)."""
        for start in range(self._held(layer), upto, self.block_size):
            n = min(self.block_size, upto - start)
            blk = self._new_block(layer, start)
            blk.gpu_data[0, :, :n] = key[0, :, start:start + n]
            blk.gpu_data[1, :, :n] = value[0, :, start:start + n]
            blk.token_count = n

    def ingest_step(self, past_key_values) -> None:
        """Take in the KV cache of a forward pass (positions not yet managed)."""
        layers = self._to_legacy(past_key_values)
        for layer, (key, value) in enumerate(layers):
            self._absorb_range(layer, key, value, key.shape[2])
        self._total_tokens = layers[0][0].shape[2]

    def append_token(self, past_key_values) -> None:
        """Take in only the newest position of every layer (one token, however
        many positions the cache is ahead)."""
        layers = self._to_legacy(past_key_values)
        for layer, (key, value) in enumerate(layers):
            if not self._blocks[layer]:
                self._absorb_range(layer, key, value, key.shape[2])
                continue
            held = self._held(layer)
            if key.shape[2] <= held:
                continue
            tail = self._blocks[layer][-1]
            if tail.token_count == tail.capacity:
                tail = self._new_block(layer, held)
            elif tail.tier != TIER_GPU:
                self._promote_block(tail)
            slot = tail.token_count
            tail.gpu_data[0, :, slot] = key[0, :, -1]
            tail.gpu_data[1, :, slot] = value[0, :, -1]
            tail.token_count = slot + 1
        self._total_tokens = layers[0][0].shape[2]

    # -- build -------------------------------------------------------------------------
    def build_past_kv(self, device: str = "cuda"):
        """past_key_values of every managed position, promoting blocks that are
        not on the GPU first."""
        per_layer = []
        for layer in range(self.n_layers):
            live = [b for b in self._blocks[layer] if b.token_count > 0]
            for b in live:
                if b.tier != TIER_GPU:
                    self._promote_block(b)
            if live:
                kv = [torch.cat([b.gpu_data[half, :, :b.token_count] for b in live], dim=1)
                      .unsqueeze(0).to(device) for half in (0, 1)]
            else:
                kv = [torch.zeros(1, self.n_kv_heads, 0, self.head_dim, dtype=self.dtype,
                                  device=device) for _ in (0, 1)]
            per_layer.append(tuple(kv))
        return self._from_legacy(tuple(per_layer))

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
        """One cycle: the GPU usage to the manager and its schedule pass, then
        the manager-side moves decided from the usage measured before them."""
        if self._tm_handle is None:
            return {}
        budget = self.gpu_budget_bytes
        used = self.gpu_kv_bytes()
        ratio = min(used / budget, 1.0) if budget > 0 else 0.0
        self._bind_stream()
        self._C.tm_set_usage(self._tm_handle, ratio, 0.0)
        self._C.tm_schedule_once(self._tm_handle)
        tm_stats = self._C.tm_get_stats(self._tm_handle)
        evicted = self._evict_cold_blocks() if budget > 0 and used > budget * _EVICT_ABOVE else 0
        if self.ssd_dir:
            self._spill_dram_to_ssd()
        promoted = (self._promote_warm_blocks()
                    if budget > 0 and used < budget * _PROMOTE_BELOW else 0)
        return {"step": self._step, "gpu_kv_bytes": used, "gpu_ratio": ratio,
                "evicted": evicted, "promoted": promoted, "tm_stats": tm_stats}

    def _ranked(self, tier: int, holder: str, *, most_accessed_first: bool = False,
                skip_sinks: bool = False) -> list[KVBlock]:
        """Blocks on `tier` whose `holder` tensor exists, by access count (ties
        keep layer-then-token order)."""
        found = [b for b in self._every_block() if b.tier == tier
                 and getattr(b, holder) is not None and not (skip_sinks and b.is_sink)]
        return sorted(found, key=attrgetter("access_count"), reverse=most_accessed_first)

    def _evict_cold_blocks(self, max_evict: int = 8) -> int:
        """Least-accessed non-sink GPU blocks to DRAM, while the GPU holds more
        than 70% of the budget."""
        moved = 0
        for blk in self._ranked(TIER_GPU, "gpu_data", skip_sinks=True)[:max_evict]:
            if self.gpu_budget_bytes > 0 and \
                    self.gpu_kv_bytes() <= self.gpu_budget_bytes * _EVICT_DOWN_TO:
                break
            self._demote_block(blk)
            moved += 1
        return moved

    def _promote_warm_blocks(self, max_promote: int = 4) -> int:
        """Most-accessed DRAM blocks back to the GPU."""
        chosen = self._ranked(TIER_DRAM, "dram_data", most_accessed_first=True)[:max_promote]
        for blk in chosen:
            self._promote_block(blk)
        return len(chosen)

    def _spill_dram_to_ssd(self, max_spill: int = 4):
        """Least-accessed non-sink DRAM blocks to files, once at least four
        such blocks are in DRAM."""
        ranked = self._ranked(TIER_DRAM, "dram_data", skip_sinks=True)
        if len(ranked) >= 4:
            for blk in ranked[:max_spill]:
                self._save_to_ssd(blk)

    # -- tier moves ---------------------------------------------------------------------------
    def _file_of(self, blk: KVBlock) -> str:
        return os.path.join(self.ssd_dir, f"blk_{blk.block_id}.bin")

    def _relocate(self, blk: KVBlock, dest: int):
        """Move one block's bytes one tier (GPU <-> pinned DRAM <-> file), count
        the move and record the new tier with the tracker where the reference
        does.  A promoted block keeps its pinned copy for its next demotion."""
        src = blk.tier
        if (src, dest) == (TIER_GPU, TIER_DRAM):
            if blk.dram_data is None:
                blk.dram_data = torch.empty(self._shape, dtype=self.dtype, pin_memory=True)
            blk.dram_data.copy_(blk.gpu_data)
            blk.gpu_data = None
        elif (src, dest) == (TIER_DRAM, TIER_GPU):
            blk.gpu_data = blk.dram_data.to("cuda")
        elif (src, dest) == (TIER_DRAM, TIER_SSD):
            blk.ssd_path = self._file_of(blk)
            with open(blk.ssd_path, "wb") as fh:          # the tensor's raw bytes
                fh.write(blk.dram_data.contiguous().view(torch.uint8).numpy().tobytes())
            blk.dram_data = None
        elif (src, dest) == (TIER_SSD, TIER_DRAM):
            with open(blk.ssd_path, "rb") as fh:
                raw = torch.frombuffer(bytearray(fh.read()), dtype=torch.uint8)
            blk.dram_data = raw.view(self.dtype).reshape(self._shape).clone().pin_memory()
        else:
            raise ValueError(f"no move from tier {src} to tier {dest}")
        blk.tier = dest
        self._moves[_MOVES[(src, dest)]] += 1
        if self._tm_handle is not None and (dest != TIER_DRAM or src == TIER_GPU):
            tier = {TIER_GPU: self._C.GPU_HBM, TIER_DRAM: self._C.HOST_DRAM,
                    TIER_SSD: self._C.SSD}[dest]
            self._C.tm_set_block_tier(self._tm_handle, blk.block_id, int(tier))

    def _demote_block(self, blk: KVBlock):
        if blk.tier == TIER_GPU and blk.gpu_data is not None:
            self._relocate(blk, TIER_DRAM)

    def _promote_block(self, blk: KVBlock):
        """To the GPU, through DRAM for a block in a file (a missing file
        leaves the block where it is)."""
        if blk.tier == TIER_SSD and blk.ssd_path is not None and os.path.exists(blk.ssd_path):
            self._relocate(blk, TIER_DRAM)
        if blk.tier == TIER_DRAM and blk.dram_data is not None:
            self._relocate(blk, TIER_GPU)

    def _save_to_ssd(self, blk: KVBlock):
        if self.ssd_dir is not None and blk.dram_data is not None:
            self._relocate(blk, TIER_SSD)

    # -- statistics -----------------------------------------------------------------------
    def get_stats(self) -> dict:
        n = self._tier_counts()
        gpu, dram, ssd = n[TIER_GPU], n[TIER_DRAM], n[TIER_SSD]
        migrations = {name: self._moves[name] for name in _MOVES.values()}
        migrations["total_blocks"] = self._ids
        tm_stats = self._C.tm_get_stats(self._tm_handle) if self._tm_handle is not None else {}
        return {"step": self._step, "total_tokens": self._total_tokens,
                "blocks_gpu": gpu, "blocks_dram": dram, "blocks_ssd": ssd,
                "blocks_total": gpu + dram + ssd,
                "gpu_kv_mb": gpu * self._block_bytes / (1 << 20),
                "dram_kv_mb": dram * self._block_bytes / (1 << 20),
                "migrations": migrations, "tm": tm_stats}

    def __repr__(self) -> str:
        s = self.get_stats()
        tiers = " ".join(f"{_TIER_NAMES[t]}:{s['blocks_' + _TIER_NAMES[t].lower()]}"
                         for t in (TIER_GPU, TIER_DRAM, TIER_SSD))
        return (f"KVCacheManager(tokens={s['total_tokens']}, blocks={s['blocks_total']} "
                f"[{tiers}], gpu_kv={s['gpu_kv_mb']:.1f}MB)")
