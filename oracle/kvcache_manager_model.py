"""The reference's KVCacheManager restated on the oracle tracker.

TEST INFRASTRUCTURE ONLY: the model the B200 KVCacheManager is compared
with.  It follows python/orchkv/kvcache_manager.py (the reference's
block-level manager) decision for decision -- block allocation and sink
flags (:144-163), ingest and append (:197-268), rebuild (:270-315), the
block-ordered report of per-block attention mass (:317-347), schedule's
thresholds at 85% / 60% of the budget (:355-397), eviction by access count
until 70% (:399-427), promotion (:429-448), spills once 4 DRAM blocks exist
(:450-463), tier bookkeeping of the manager's tracker (:465-529) -- with
the orchkv_core calls going to the
oracle tracker and block data kept as numpy arrays on the host.  Mass per
block is float(avg[:, s:e].sum()) on the caller's torch tensor, as the
reference computes it.
"""
from __future__ import annotations

import numpy as np

from . import oracle as O

GPU, DRAM, SSD = 0, 1, 2              # the manager's own tier numbers
TM_GPU, TM_DRAM, TM_SSD = 0, 1, 3     # StorageTier values it passes to the tracker


class ModelBlock:
    def __init__(self, bid, layer, start, cap, sink):
        self.block_id, self.layer, self.token_start = bid, layer, start
        self.token_count, self.capacity, self.is_sink = 0, cap, sink
        self.tier, self.access_count = GPU, 0
        self.data = None            # numpy [2, H, block_size, d] wherever the block lives
        self.file_bytes = None      # what a spill wrote


class ModelKVManager:
    def __init__(self, n_layers, n_kv_heads, head_dim, block_size, np_dtype, gpu_budget_bytes,
                 with_ssd, sink_tokens, tracker_cap):
        self.L, self.H, self.d, self.bs = n_layers, n_kv_heads, head_dim, block_size
        self.np_dtype = np_dtype
        self.budget, self.with_ssd, self.sink_tokens = gpu_budget_bytes, with_ssd, sink_tokens
        self.block_bytes = 2 * n_kv_heads * block_size * head_dim * np.dtype(np_dtype).itemsize
        self.blocks = [[] for _ in range(n_layers)]
        self.next_id = 0
        self.total_tokens = 0
        self.step = 0
        self.stats = {"gpu_to_dram": 0, "dram_to_gpu": 0, "dram_to_ssd": 0, "ssd_to_dram": 0,
                      "total_blocks": 0}
        self.tm = O.OracleTM(tracker_cap=tracker_cap)

    def all_blocks(self):
        for lb in self.blocks:
            yield from lb

    def gpu_kv_bytes(self):
        return sum(1 for b in self.all_blocks() if b.tier == GPU) * self.block_bytes

    def _alloc(self, layer, start):
        b = ModelBlock(self.next_id, layer, start, self.bs, start < self.sink_tokens)
        self.next_id += 1
        self.blocks[layer].append(b)
        self.stats["total_blocks"] += 1
        self.tm.register(b.block_id, 1 if b.is_sink else 0, TM_GPU)  # binding's positional order
        return b

    def _ingest_layer(self, layer, k, v, seq_len):
        have = sum(b.token_count for b in self.blocks[layer])
        for pos in range(have, seq_len, self.bs):
            end = min(pos + self.bs, seq_len)
            b = self._alloc(layer, pos)
            b.token_count = end - pos
            b.data = np.zeros((2, self.H, self.bs, self.d), self.np_dtype)
            b.data[0, :, :end - pos] = k[:, pos:end]
            b.data[1, :, :end - pos] = v[:, pos:end]

    def ingest_step(self, kv):
        """kv: list over layers of numpy (k [H, T, d], v [H, T, d])."""
        for layer, (k, v) in enumerate(kv):
            self._ingest_layer(layer, k, v, k.shape[1])
        self.total_tokens = kv[0][0].shape[1]

    def append_token(self, kv):
        for layer, (k, v) in enumerate(kv):
            seq_len = k.shape[1]
            blocks = self.blocks[layer]
            if not blocks:
                self._ingest_layer(layer, k, v, seq_len)
                continue
            have = sum(b.token_count for b in blocks)
            if seq_len <= have:
                continue
            last = blocks[-1]
            if last.token_count < last.capacity:
                if last.tier != GPU:
                    self._promote(last)
                last.data[0, :, last.token_count] = k[:, -1]
                last.data[1, :, last.token_count] = v[:, -1]
                last.token_count += 1
            else:
                b = self._alloc(layer, have)
                b.token_count = 1
                b.data = np.zeros((2, self.H, self.bs, self.d), self.np_dtype)
                b.data[0, :, 0] = k[:, -1]
                b.data[1, :, 0] = v[:, -1]
        self.total_tokens = kv[0][0].shape[1]

    def build_past_kv(self):
        out = []
        for layer in range(self.L):
            ks, vs = [], []
            for b in self.blocks[layer]:
                if b.token_count == 0:
                    continue
                if b.tier != GPU:
                    self._promote(b)
                ks.append(b.data[0, :, :b.token_count])
                vs.append(b.data[1, :, :b.token_count])
            if not ks:
                e = np.zeros((self.H, 0, self.d), self.np_dtype)
                out.append((e, e.copy()))
            else:
                out.append((np.concatenate(ks, axis=1), np.concatenate(vs, axis=1)))
        return out

    def report_attention(self, layer, avg):
        """avg: the caller's torch tensor attn.float().mean(dim=(0, 2))."""
        kv_len = avg.shape[-1]
        for b in self.blocks[layer]:
            s, e = b.token_start, min(b.token_start + b.token_count, kv_len)
            if s >= e:
                continue
            self.tm.report(b.block_id, float(avg[:, s:e].sum()))
            b.access_count += 1

    def step_done(self):
        self.step += 1
        self.tm.step_done()

    def schedule(self):
        gpu_bytes = self.gpu_kv_bytes()
        ratio = min(gpu_bytes / self.budget, 1.0) if self.budget > 0 else 0.0
        self.tm.set_usage(ratio, 0.0)
        self.tm.schedule_once()
        evicted = promoted = 0
        if self.budget > 0 and gpu_bytes > self.budget * 0.85:
            cands = [b for b in self.all_blocks() if b.tier == GPU and not b.is_sink]
            cands.sort(key=lambda b: b.access_count)
            for b in cands[:8]:
                if self.gpu_kv_bytes() <= self.budget * 0.7:
                    break
                self._demote(b)
                evicted += 1
        if self.with_ssd:
            dram = [b for b in self.all_blocks() if b.tier == DRAM and not b.is_sink]
            if len(dram) >= 4:
                dram.sort(key=lambda b: b.access_count)
                for b in dram[:4]:
                    b.file_bytes = b.data.tobytes()
                    b.tier = SSD
                    self.stats["dram_to_ssd"] += 1
                    self.tm.set_block_tier(b.block_id, TM_SSD)
        if self.budget > 0 and gpu_bytes < self.budget * 0.60:
            cands = [b for b in self.all_blocks() if b.tier == DRAM]
            cands.sort(key=lambda b: b.access_count, reverse=True)
            for b in cands[:4]:
                self._promote(b)
                promoted += 1
        return {"step": self.step, "gpu_kv_bytes": gpu_bytes, "gpu_ratio": ratio,
                "evicted": evicted, "promoted": promoted}

    def _demote(self, b):
        b.tier = DRAM
        self.stats["gpu_to_dram"] += 1
        self.tm.set_block_tier(b.block_id, TM_DRAM)

    def _promote(self, b):
        if b.tier == SSD:
            b.tier = DRAM
            self.stats["ssd_to_dram"] += 1
        if b.tier == DRAM:
            b.tier = GPU
            self.stats["dram_to_gpu"] += 1
            self.tm.set_block_tier(b.block_id, TM_GPU)

    def get_stats(self):
        n = [0, 0, 0]
        for b in self.all_blocks():
            n[b.tier] += 1
        return {"step": self.step, "total_tokens": self.total_tokens, "blocks_gpu": n[0],
                "blocks_dram": n[1], "blocks_ssd": n[2], "blocks_total": sum(n),
                "gpu_kv_mb": n[0] * self.block_bytes / (1 << 20),
                "dram_kv_mb": n[1] * self.block_bytes / (1 << 20),
                "migrations": dict(self.stats)}
