"""Test infrastructure only: a CPU restatement of the reference's
FastKVCacheManager (python/orchkv/fast_kvcache_manager.py), used as the
oracle for orchkv_b200.fast_manager.  Buffers are numpy arrays, the tiered
manager is the oracle's OracleTM (the reference's scheduler restated and
pinned against it), and every per-block loop is kept as the reference
writes it.  Nothing in the product imports this module.
"""
from __future__ import annotations

import numpy as np

from oracle.oracle import OracleTM


class FastManagerModel:
    """fast_kvcache_manager.py:53-104 (state), CPU arrays instead of CUDA."""

    def __init__(self, n_layers, n_kv_heads, head_dim, block_size=16, dtype=np.float16,
                 gpu_budget_bytes=0, max_seq_len=4096, sink_tokens=4):
        self.n_layers, self.n_kv_heads, self.head_dim = n_layers, n_kv_heads, head_dim
        self.block_size, self.dtype = block_size, np.dtype(dtype)
        self.gpu_budget_bytes, self.max_seq_len, self.sink_tokens = (gpu_budget_bytes,
                                                                     max_seq_len, sink_tokens)
        self._block_bytes = 2 * n_kv_heads * block_size * head_dim * self.dtype.itemsize
        self._total_tokens = 0
        self._step = 0
        self.k = [np.zeros((n_kv_heads, max_seq_len, head_dim), self.dtype)
                  for _ in range(n_layers)]
        self.v = [np.zeros((n_kv_heads, max_seq_len, head_dim), self.dtype)
                  for _ in range(n_layers)]
        self._evicted_ranges = [[] for _ in range(n_layers)]
        self._dram_store = {}
        self._stats = {"gpu_to_dram": 0, "dram_to_gpu": 0, "dram_to_ssd": 0, "ssd_to_dram": 0,
                       "total_blocks": 0, "evictions_this_step": 0}
        # _C.tm_create() with the binding's defaults (bindings/orchkv_pybind.cpp:215-271)
        self.tm = OracleTM()

    def gpu_kv_bytes(self):                                   # :120-123
        n_blocks = (self._total_tokens + self.block_size - 1) // self.block_size
        evicted = sum(len(e) for e in self._evicted_ranges)
        return (n_blocks * self.n_layers - evicted) * self._block_bytes

    def ingest(self, k_layers, v_layers):                     # :141-156
        seq_len = k_layers[0].shape[1]
        for li in range(self.n_layers):
            self.k[li][:, :seq_len] = k_layers[li]
            self.v[li][:, :seq_len] = v_layers[li]
        self._total_tokens = seq_len
        n_blocks = (seq_len + self.block_size - 1) // self.block_size
        for bid in range(n_blocks):
            flags = 1 if (bid * self.block_size) < self.sink_tokens else 0
            self.tm.register(bid, flags, 0)                   # positional: tier := flags
        self._stats["total_blocks"] = n_blocks * self.n_layers

    def append(self, k_tok, v_tok):                           # :158-173
        pos = self._total_tokens
        for li in range(self.n_layers):
            self.k[li][:, pos] = k_tok[li]
            self.v[li][:, pos] = v_tok[li]
        self._total_tokens = pos + 1
        if pos % self.block_size == 0:
            flags = 1 if pos < self.sink_tokens else 0
            self.tm.register(pos // self.block_size, flags, 0)

    def restore(self):                                        # :204-219
        for li in range(self.n_layers):
            for (start, end) in self._evicted_ranges[li]:
                key = (li, start, end)
                if key in self._dram_store:
                    kd, vd = self._dram_store.pop(key)
                    self.k[li][:, start:end] = kd
                    self.v[li][:, start:end] = vd
                    self._stats["dram_to_gpu"] += 1
            self._evicted_ranges[li].clear()

    def report_attention(self, avg):                          # :221-235, avg [q-heads, T]
        n_blocks = (self._total_tokens + self.block_size - 1) // self.block_size
        for bid in range(n_blocks):
            start = bid * self.block_size
            end = min(start + self.block_size, self._total_tokens)
            if start >= avg.shape[-1]:
                break
            end = min(end, avg.shape[-1])
            score = float(np.sum(avg[:, start:end], dtype=np.float32))
            self.tm.report(bid, score)

    def step_done(self):                                      # :272-275
        self._step += 1
        self.tm.step_done()

    def schedule(self):                                       # :277-298
        n_blocks = (self._total_tokens + self.block_size - 1) // self.block_size
        evicted_count = sum(len(e) for e in self._evicted_ranges)
        total = n_blocks * self.n_layers
        gpu_ratio = 1.0 - evicted_count / total if total > 0 else 0.0
        self.tm.set_usage(gpu_ratio, 0.0)
        self.tm.schedule_once()
        self._stats["evictions_this_step"] = 0
        if self.gpu_budget_bytes > 0 and self.gpu_kv_bytes() > self.gpu_budget_bytes * 0.85:
            self._evict_cold_blocks()
        return {"step": self._step, "gpu_ratio": gpu_ratio}

    def _evict_cold_blocks(self, max_evict=8):                # :300-345
        n_blocks = (self._total_tokens + self.block_size - 1) // self.block_size
        evicted_bids = set()
        for ranges in self._evicted_ranges:
            for (s, e) in ranges:
                evicted_bids.add(s // self.block_size)
        candidates = [bid for bid in range(n_blocks)
                      if bid not in evicted_bids and bid * self.block_size >= self.sink_tokens]
        candidates.sort(key=lambda bid: float(self.tm.score(bid)))
        evicted = 0
        for bid in candidates[:max_evict]:
            start = bid * self.block_size
            end = min(start + self.block_size, self._total_tokens)
            for li in range(self.n_layers):
                self._dram_store[(li, start, end)] = (self.k[li][:, start:end].copy(),
                                                      self.v[li][:, start:end].copy())
                self._evicted_ranges[li].append((start, end))
                self._stats["gpu_to_dram"] += 1
            evicted += 1
            self._stats["evictions_this_step"] += 1
            if self.gpu_kv_bytes() <= self.gpu_budget_bytes * 0.85:
                break
        return evicted

    def evicted_blocks(self):
        return sorted({s // self.block_size for s, _ in self._evicted_ranges[0]})

    def get_stats(self):                                      # :347-360
        n_blocks = (self._total_tokens + self.block_size - 1) // self.block_size
        evicted = sum(len(e) for e in self._evicted_ranges)
        gpu_blocks = n_blocks * self.n_layers - evicted
        return {"step": self._step, "total_tokens": self._total_tokens,
                "blocks_gpu": gpu_blocks, "blocks_dram": evicted, "blocks_ssd": 0,
                "blocks_total": n_blocks * self.n_layers,
                "gpu_kv_mb": gpu_blocks * self._block_bytes / (1 << 20),
                "migrations": dict(self._stats)}
