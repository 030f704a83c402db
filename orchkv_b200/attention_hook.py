"""Attention-score collection for decode loops, on the GPU end to end.

Same interface and behaviour as the reference's
python/orchkv/vllm_integration/attention_hook.py (AttentionScoreCollector,
AttentionHookManager): every `sample_interval` steps each layer's attention
weights [batch, heads, q_len, kv_len] are reduced to one score per (head,
block) -- the mean over batch, query positions and the block's token
positions, the last block padded with zeros (attention_hook.py:118-140) --
and each score is reported to the tiered manager for block id
block_id_fn(layer, head, block), else block_table[0, block], else
layer * heads * n_blocks + head * n_blocks + block (attention_hook.py:155-189).

The reference reduces on a side stream, copies the scores to pinned host
memory, synchronises and calls tm_report_attn once per block from Python.
Here one call, tm_report_attn_blockmean, reduces and records every report on
the device in the reference's order (heads of a block in head order), so a
sampled layer costs two kernel launches and no host round trip.  Reports
whose ids would make two blocks share a tracker slot take the same device
reduction and then one device batch of reports in the hook's order, whose
shared slots are applied in list order; only an id whose low 32 bits equal
the device's no-block marker still goes through tm_report_attn one by one.

The manager handle is an ``orchkv_core.tm_create`` handle, as in the
reference; the manager's GPU work runs on torch's current stream.
"""
from __future__ import annotations

import logging
from typing import Any, Callable

import numpy as np
import torch

from . import core

logger = logging.getLogger(__name__)

_DTYPES = {torch.float16: 0, torch.bfloat16: 1, torch.float32: 2}
_NO_BLOCK = 0xFFFFFFFF


class AttentionScoreCollector:
    """Per-block attention scores of sampled decode steps, fed to a tiered
    manager (reference: attention_hook.py:33-215)."""

    def __init__(self, tm_handle: int, block_size: int = 16, sample_interval: int = 10):
        self._C = core()
        self._tm = tm_handle
        self._block_size = block_size
        self._sample_interval = max(1, sample_interval)
        self._step = 0
        self._enabled = True
        self._tm_stream = None
        self._cap = int(self._C.tm_capacity(tm_handle))
        self._stats = {"samples_taken": 0, "blocks_reported": 0, "steps_skipped": 0}

    # -- configuration ------------------------------------------------------
    @property
    def block_size(self) -> int:
        return self._block_size

    @property
    def sample_interval(self) -> int:
        return self._sample_interval

    @sample_interval.setter
    def sample_interval(self, v: int):
        self._sample_interval = max(1, v)

    def should_sample(self) -> bool:
        """Steps 0, k, 2k, ... are sampled while enabled."""
        return self._enabled and self._step % self._sample_interval == 0

    def set_enabled(self, enabled: bool):
        self._enabled = enabled

    # -- device work ----------------------------------------------------------
    def _bind_stream(self):
        s = torch.cuda.current_stream().cuda_stream
        if s != self._tm_stream:
            self._C.tm_set_stream(self._tm, s)
            self._tm_stream = s

    def _weights(self, attn_weights: torch.Tensor):
        if attn_weights.dim() != 4 or not attn_weights.is_cuda:
            raise ValueError("attention weights must be a CUDA tensor "
                             "[batch, heads, q_len, kv_len]")
        dt = _DTYPES.get(attn_weights.dtype)
        if dt is None:
            attn_weights, dt = attn_weights.float(), 2
        return attn_weights.contiguous(), dt

    def _reduce(self, w: torch.Tensor, dt: int, ids: torch.Tensor | None) -> torch.Tensor:
        bs, heads, q_len, kv_len = w.shape
        nb = (kv_len + self._block_size - 1) // self._block_size
        scores = torch.empty(heads, nb, dtype=torch.float32, device=w.device)
        self._bind_stream()
        rc = self._C.tm_report_attn_blockmean(
            self._tm, w.data_ptr(), dt, bs, heads, q_len, kv_len, self._block_size,
            0 if ids is None else ids.data_ptr(), scores.data_ptr())
        if rc != 0:
            raise RuntimeError(f"tm_report_attn_blockmean failed: {rc}")
        return scores

    def _blockwise_reduce(self, attn_weights: torch.Tensor, n_blocks: int) -> torch.Tensor:
        """[batch, heads, q_len, kv_len] -> [heads, n_blocks] block means, in the
        weights' dtype (attention_hook.py:118-140)."""
        w, dt = self._weights(attn_weights)
        kv_len = w.shape[3]
        if n_blocks * self._block_size < kv_len:
            raise ValueError(f"{n_blocks} blocks of {self._block_size} do not cover "
                             f"{kv_len} positions")
        scores = self._reduce(w, dt, None)
        if scores.shape[1] < n_blocks:           # blocks wholly past kv_len: zeros
            pad = torch.zeros(scores.shape[0], n_blocks - scores.shape[1],
                              dtype=scores.dtype, device=scores.device)
            scores = torch.cat([scores, pad], dim=1)
        return scores.to(attn_weights.dtype)

    def _block_ids(self, layer_idx, heads, n_blocks, block_table, block_id_fn) -> np.ndarray:
        """int64 [heads, n_blocks] of report ids, -1 where nothing is reported,
        chosen as the reference chooses them (attention_hook.py:171-182)."""
        ids = np.full((heads, n_blocks), -1, np.int64)
        if block_id_fn is not None:
            for h in range(heads):
                for bi in range(n_blocks):
                    bid = block_id_fn(layer_idx, h, bi)
                    if bid is not None and bid >= 0:
                        ids[h, bi] = bid
            return ids
        col = np.arange(n_blocks, dtype=np.int64)
        ids[:] = layer_idx * heads * n_blocks + np.arange(heads, dtype=np.int64)[:, None] * \
            n_blocks + col[None, :]
        if block_table is not None:
            width = min(int(block_table.shape[-1]), n_blocks)
            row = np.asarray(block_table[0, :width].tolist(), np.int64)
            ids[:, :width] = row[None, :]
            ids[ids < 0] = -1
        return ids

    def _device_order_ok(self, ids: np.ndarray) -> bool:
        """The device records a block's heads in order and blocks in parallel:
        exact when no tracker slot is shared by two blocks and no id's low
        32 bits are the no-block marker."""
        valid = ids >= 0
        if not valid.any():
            return True
        v = ids[valid]
        if np.any((v & 0xFFFFFFFF) == _NO_BLOCK):
            return False
        slots = v & (self._cap - 1)
        cols = np.nonzero(valid)[1]
        pairs = np.unique(slots * ids.shape[1] + cols)
        return len(np.unique(pairs // ids.shape[1])) == len(pairs)

    def collect(self, layer_idx: int, attn_weights: torch.Tensor,
                block_table: torch.Tensor | None = None,
                block_id_fn: Callable[[int, int, int], int | None] | None = None):
        """Reduce one layer's attention weights and report them (sampled steps
        only)."""
        if not self.should_sample():
            return
        w, dt = self._weights(attn_weights)
        bs, heads, q_len, kv_len = w.shape
        nb = (kv_len + self._block_size - 1) // self._block_size
        ids = self._block_ids(layer_idx, heads, nb, block_table, block_id_fn)
        valid = ids >= 0
        if self._device_order_ok(ids):
            ids32 = np.where(valid, ids & 0xFFFFFFFF, _NO_BLOCK).astype(np.uint32)
            ids_d = torch.from_numpy(ids32.view(np.int32)).to(w.device)
            self._reduce(w, dt, ids_d)
        elif not np.any((ids[valid] & 0xFFFFFFFF) == _NO_BLOCK):
            # blocks sharing tracker slots: the scores' reports in the hook's
            # order (head by head, block by block) as one device batch, which
            # applies a shared slot's reports in list order, as that many
            # tm_report_attn calls would
            scores = self._reduce(w, dt, None)
            flat = np.flatnonzero(valid.reshape(-1))
            ids_d = torch.from_numpy((ids.reshape(-1)[flat] & 0xFFFFFFFF).astype(np.uint32)
                                     .view(np.int32)).to(w.device)
            w_d = scores.reshape(-1)[torch.from_numpy(flat).to(w.device)].contiguous()
            rc = self._C.tm_report_attn_batch_dev(self._tm, ids_d.data_ptr(), w_d.data_ptr(),
                                                  len(flat))
            if rc != 0:
                raise RuntimeError(f"tm_report_attn_batch_dev failed: {rc}")
        else:
            # an id whose low 32 bits are the device's no-block marker: one
            # report at a time through the per-block call
            scores = self._reduce(w, dt, None).cpu()
            for h in range(heads):
                for bi in range(nb):
                    if valid[h, bi]:
                        self._C.tm_report_attn(self._tm, int(ids[h, bi]), float(scores[h, bi]))
        self._stats["blocks_reported"] += int(valid.sum())

    def on_step_done(self):
        """End of a decode step: advance the step and the manager's tracker
        (attention_hook.py:191-207)."""
        self._step += 1
        if self.should_sample():
            self._stats["samples_taken"] += 1
        else:
            self._stats["steps_skipped"] += 1
        self._bind_stream()
        self._C.tm_step_done(self._tm)

    def get_stats(self) -> dict[str, Any]:
        return {**self._stats, "current_step": self._step,
                "sample_interval": self._sample_interval, "block_size": self._block_size,
                "enabled": self._enabled}


class AttentionHookManager:
    """Wraps a model's self-attention modules so that sampled steps return
    attention weights and feed them to the collector (reference:
    attention_hook.py:218-377)."""

    def __init__(self, collector: AttentionScoreCollector, attn_module_name: str = "attn"):
        self._collector = collector
        self._attn_module_name = attn_module_name
        self._original_forwards: dict[int, Callable] = {}
        self._modules: dict[int, torch.nn.Module] = {}
        self._layer_map: dict[int, int] = {}
        self._installed = False

    def install(self, model: torch.nn.Module):
        """Wrap every module whose name contains both the attention name and
        'self_attn', numbering them as layers in model order."""
        if self._installed:
            logger.warning("AttentionHookManager already installed")
            return
        layer = 0
        for name, module in model.named_modules():
            if self._is_attention_module(name, module):
                self._wrap_module(module, layer)
                self._layer_map[id(module)] = layer
                layer += 1
        self._installed = True
        logger.info("AttentionHookManager: installed hooks on %d layers", layer)

    def _is_attention_module(self, name: str, module: torch.nn.Module) -> bool:
        low = name.lower()
        return self._attn_module_name in low and "self_attn" in low

    def _wrap_module(self, module: torch.nn.Module, layer_idx: int):
        original = module.forward
        self._original_forwards[id(module)] = original
        self._modules[id(module)] = module
        collector = self._collector

        def hooked_forward(*args, **kwargs):
            sample = collector.should_sample()
            if sample:
                kwargs["output_attentions"] = True
            result = original(*args, **kwargs)
            if sample:
                weights = self._extract_attn_weights(result, kwargs)
                if weights is not None:
                    collector.collect(layer_idx=layer_idx, attn_weights=weights,
                                      block_table=kwargs.get("block_table"))
            return result

        module.forward = hooked_forward

    @staticmethod
    def _extract_attn_weights(result: Any, kwargs: dict) -> torch.Tensor | None:
        """Weights from (output, weights, ...) or a dict's attn_weights /
        attention_weights / attentions entry."""
        if isinstance(result, tuple) and len(result) >= 2:
            cand = result[1]
            if isinstance(cand, torch.Tensor) and cand.dim() == 4:
                return cand
        if isinstance(result, dict):
            for key in ("attn_weights", "attention_weights", "attentions"):
                if isinstance(result.get(key), torch.Tensor):
                    return result[key]
        return None

    def on_step_done(self):
        self._collector.on_step_done()

    def uninstall(self):
        """Put every wrapped module's own forward back."""
        for key, original in self._original_forwards.items():
            self._modules[key].forward = original
        self._original_forwards.clear()
        self._modules.clear()
        self._layer_map.clear()
        self._installed = False

    @property
    def collector(self) -> AttentionScoreCollector:
        return self._collector

    def get_stats(self) -> dict[str, Any]:
        return {"installed": self._installed, "n_layers_hooked": len(self._layer_map),
                "collector": self._collector.get_stats()}
