"""vLLM V1 KV connector on the B200 path.

The reference's python/orchkv/vllm_integration/connector.py with the same
classes, methods, metadata and statistics; the worker's data plane is
batched: a layer's save is one copy launch gathering every listed block of
the layer's cache tensor into a pinned store, a layer's load one launch
scattering them back (the reference: one ``copy_`` per block and layer,
connector.py:136-195).  The scheduler side is the reference's bookkeeping
(connector.py:220-282), unchanged in behaviour.

Cache tensors are indexed by block along dim 0 (``kv_layer[block_id]``), as
the reference assumes; a layer whose blocks are not contiguous chunks falls
back to per-block copies.
"""
from __future__ import annotations

import logging
import threading
from dataclasses import dataclass, field
from typing import Any

import torch

from . import core

logger = logging.getLogger(__name__)

try:
    from vllm.distributed.kv_transfer.kv_connector.v1.base import (
        KVConnectorBase_V1,
        KVConnectorMetadata,
        KVConnectorRole,
    )
    HAS_VLLM = True
except ImportError:  # pragma: no cover - vLLM is part of the image
    HAS_VLLM = False

    class KVConnectorRole:
        SCHEDULER = "scheduler"
        WORKER = "worker"

    class KVConnectorMetadata:
        pass

    class KVConnectorBase_V1:
        """Stand-in with the base class's metadata plumbing."""

        def __init__(self, vllm_config, role, kv_cache_config=None):
            self._connector_metadata = None
            self._role = role

        @property
        def role(self):
            return self._role

        def bind_connector_metadata(self, meta):
            self._connector_metadata = meta

        def clear_connector_metadata(self):
            self._connector_metadata = None


@dataclass
class OrchKvConnectorMetadata(KVConnectorMetadata):
    """Metadata passed from scheduler to worker each step."""
    blocks_to_save: dict[str, list[int]] = field(default_factory=dict)
    blocks_to_load: dict[str, list[int]] = field(default_factory=dict)
    req_block_map: dict[str, dict[int, int]] = field(default_factory=dict)


class _LayerStore:
    """Pinned slots holding saved blocks of one layer: block id -> slot."""

    def __init__(self, block_elems: int, dtype: torch.dtype):
        self.block_elems, self.dtype = block_elems, dtype
        self.buf = None
        self.slot: dict[int, int] = {}
        self.free: list[int] = []

    def slots_for(self, block_ids: list[int], streams) -> list[int]:
        out = []
        for bid in block_ids:
            s = self.slot.get(bid)
            if s is None:
                s = self.free.pop() if self.free else len(self.slot)
                self.slot[bid] = s
            out.append(s)
        need = max(out) + 1 if out else 0
        if self.buf is None or self.buf.shape[0] < need:
            cap = max(need, 2 * (0 if self.buf is None else self.buf.shape[0]), 16)
            new = torch.empty(cap, self.block_elems, dtype=self.dtype).pin_memory()
            if self.buf is not None:
                for st in streams:                   # copies in flight on the old buffer
                    st.synchronize()
                new[: self.buf.shape[0]].copy_(self.buf)
            self.buf = new
        return out

    def release(self, bid: int):
        s = self.slot.pop(bid, None)
        if s is not None:
            self.free.append(s)


class OrchKvConnectorWorker:
    """Worker side: batched GPU <-> pinned DRAM block copies."""

    def __init__(self, orchkv_cfg: dict[str, Any]):
        self._kv_caches: dict[str, torch.Tensor] = {}
        self._save_stream = torch.cuda.Stream()
        self._load_stream = torch.cuda.Stream()
        self._pending_saves: list[tuple[str, int]] = []
        self._pending_loads: list[tuple[str, int]] = []
        self._load_events: dict[str, torch.cuda.Event] = {}
        self._stores: dict[str, _LayerStore] = {}
        self._lock = threading.Lock()
        self._save_count = 0
        self._load_count = 0
        self._initialized = False
        self._orchkv_cfg = orchkv_cfg
        self._C = core()

    def _ensure_init(self):
        if self._initialized:
            return
        cfg = self._C.Config()
        cfg.gpu_pool_bytes = 0  # GPU memory is managed by vLLM
        cfg.dram_pool_bytes = self._orchkv_cfg.get("dram_pool_bytes", 8 * (1 << 30))
        cfg.d_head = self._orchkv_cfg.get("d_head", 128)
        cfg.tokens_per_block = self._orchkv_cfg.get("tokens_per_block", 16)
        cfg.num_cuda_streams = self._orchkv_cfg.get("num_cuda_streams", 4)
        cfg.orchfs_io_workers = self._orchkv_cfg.get("io_workers", 4)
        self._C.init(cfg)
        self._initialized = True

    def register_kv_caches(self, kv_caches: dict[str, torch.Tensor]):
        self._kv_caches = kv_caches
        self._ensure_init()
        logger.info("OrchKvConnector: registered %d KV cache layers", len(kv_caches))

    def _store(self, layer_name: str, kv_layer: torch.Tensor) -> _LayerStore:
        st = self._stores.get(layer_name)
        if st is None:
            st = _LayerStore(kv_layer[0].numel(), kv_layer.dtype)
            self._stores[layer_name] = st
        return st

    @staticmethod
    def _batched(kv_layer: torch.Tensor) -> bool:
        chunk = kv_layer[0].numel() * kv_layer.element_size()
        return (kv_layer[0].is_contiguous() and kv_layer.stride(0) == kv_layer[0].numel()
                and chunk % 16 == 0 and kv_layer.data_ptr() % 16 == 0)

    def _copy(self, kv_layer, store, block_ids, slots, direction, stream):
        chunk = kv_layer[0].numel() * kv_layer.element_size()
        dev = kv_layer.device
        ids = torch.tensor(block_ids, dtype=torch.int32).pin_memory().to(dev, non_blocking=True)
        sl = torch.tensor(slots, dtype=torch.int32).pin_memory().to(dev, non_blocking=True)
        rc = self._C.copy_token_blocks([kv_layer.data_ptr()], 1, 0, chunk, 1, kv_layer.shape[0],
                                       ids.data_ptr(), len(block_ids), store.buf.data_ptr(),
                                       direction, stream.cuda_stream, sl.data_ptr())
        if rc != 0:
            raise RuntimeError(f"orchkv_copy_token_blocks failed: {rc}")
        # keep the index tensors alive until the copy has run
        ids.record_stream(stream)
        sl.record_stream(stream)

    def save_kv_layer(self, layer_name: str, kv_layer: torch.Tensor,
                      metadata: OrchKvConnectorMetadata, block_ids: list[int] | None = None):
        """Async save: GPU -> pinned DRAM, one launch for the layer."""
        if block_ids is None:
            block_ids = metadata.blocks_to_save.get(layer_name, [])
        if not block_ids:
            return
        self._save_stream.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(self._save_stream):
            with self._lock:
                st = self._store(layer_name, kv_layer)
                slots = st.slots_for(block_ids, (self._save_stream, self._load_stream))
            if self._batched(kv_layer):
                self._copy(kv_layer, st, block_ids, slots, 0, self._save_stream)
            else:
                for bid, s in zip(block_ids, slots):
                    st.buf[s].view(kv_layer[bid].shape).copy_(kv_layer[bid], non_blocking=True)
            self._pending_saves.extend((layer_name, b) for b in block_ids)
        self._save_count += len(block_ids)

    def wait_for_save(self):
        """Block until all pending saves are complete."""
        self._save_stream.synchronize()
        self._pending_saves.clear()

    def start_load_kv(self, metadata: OrchKvConnectorMetadata):
        """Kick off async loads: pinned DRAM -> GPU, one launch per layer."""
        self._load_stream.wait_stream(torch.cuda.current_stream())
        for layer_name, block_ids in metadata.blocks_to_load.items():
            kv_layer = self._kv_caches.get(layer_name)
            if kv_layer is None:
                continue
            with self._lock:
                st = self._stores.get(layer_name)
                have = [(b, st.slot[b]) for b in block_ids if b in st.slot] if st else []
            missing = [b for b in block_ids if not st or b not in st.slot]
            for b in missing:
                logger.warning("OrchKv: no DRAM buffer for %s block %d", layer_name, b)
            with torch.cuda.stream(self._load_stream):
                if have:
                    self._load_stream.wait_stream(self._save_stream)
                    bids = [b for b, _ in have]
                    slots = [s for _, s in have]
                    if self._batched(kv_layer):
                        self._copy(kv_layer, st, bids, slots, 1, self._load_stream)
                    else:
                        for b, s in have:
                            kv_layer[b].copy_(st.buf[s].view(kv_layer[b].shape),
                                              non_blocking=True)
                    self._pending_loads.extend((layer_name, b) for b in bids)
                event = self._load_stream.record_event()
                self._load_events[layer_name] = event
        self._load_count += sum(len(b) for b in metadata.blocks_to_load.values())

    def wait_for_layer_load(self, layer_name: str):
        """Block until a specific layer's load is complete."""
        event = self._load_events.pop(layer_name, None)
        if event is not None:
            event.synchronize()

    def free_blocks(self, layer_name: str, block_ids: list[int]):
        """Release the DRAM slots of freed blocks."""
        with self._lock:
            st = self._stores.get(layer_name)
            if st:
                for b in block_ids:
                    st.release(b)

    def get_stats(self) -> dict[str, Any]:
        return {"save_count": self._save_count, "load_count": self._load_count,
                "dram_buffers": sum(len(s.slot) for s in self._stores.values())}

    def shutdown(self):
        self._save_stream.synchronize()
        self._load_stream.synchronize()
        with self._lock:
            self._stores.clear()
        if self._initialized:
            self._C.shutdown()
            self._initialized = False


class OrchKvConnectorScheduler:
    """Scheduler side: which blocks to offload / load (connector.py:220-282)."""

    def __init__(self, orchkv_cfg: dict[str, Any]):
        self._orchkv_cfg = orchkv_cfg
        self._cached_requests: dict[str, set[int]] = {}
        self._pending_offload: dict[str, list[int]] = {}
        self._pending_load: dict[str, list[int]] = {}

    def get_num_new_matched_tokens(self, request, num_computed_tokens: int):
        cached = self._cached_requests.get(request.request_id)
        if cached is None:
            return 0, False
        new_tokens = max(0, len(cached) - num_computed_tokens)
        return new_tokens, (new_tokens > 0)

    def update_state_after_alloc(self, request, blocks, num_external_tokens: int):
        pass

    def build_connector_meta(self, scheduler_output) -> OrchKvConnectorMetadata:
        meta = OrchKvConnectorMetadata()
        meta.blocks_to_save = dict(self._pending_offload)
        meta.blocks_to_load = dict(self._pending_load)
        self._pending_offload.clear()
        self._pending_load.clear()
        return meta

    def request_finished(self, request, block_ids: list[int]):
        self._cached_requests[request.request_id] = set(block_ids)
        return False, None

    def handle_preemptions(self, preempted_req_ids: set[str]):
        for req_id in preempted_req_ids:
            cached = self._cached_requests.get(req_id)
            if cached:
                for layer_name in self._get_layer_names():
                    self._pending_offload.setdefault(layer_name, []).extend(cached)

    def _get_layer_names(self) -> list[str]:
        return [f"layer_{i}" for i in range(self._orchkv_cfg.get("n_layers", 32))]


class OrchKvOffloadingConnector(KVConnectorBase_V1):
    """vLLM V1 connector routing KV offloading through the B200 data plane
    (connector.py:285-421)."""

    @property
    def prefer_cross_layer_blocks(self) -> bool:
        return True

    def __init__(self, vllm_config, role, kv_cache_config=None):
        super().__init__(vllm_config, role, kv_cache_config)
        extra_cfg = {}
        ktc = getattr(vllm_config, "kv_transfer_config", None)
        if ktc is not None and hasattr(ktc, "kv_connector_extra_config"):
            extra_cfg = ktc.kv_connector_extra_config or {}
        mc = getattr(vllm_config, "model_config", None)
        orchkv_cfg = {
            "dram_pool_bytes": int(extra_cfg.get("dram_pool_gb", 8)) * (1 << 30),
            "d_head": getattr(mc, "head_dim", extra_cfg.get("d_head", 128)),
            "tokens_per_block": extra_cfg.get("tokens_per_block", 16),
            "num_cuda_streams": extra_cfg.get("num_cuda_streams", 4),
            "io_workers": extra_cfg.get("io_workers", 4),
            "n_layers": getattr(mc, "num_layers", extra_cfg.get("n_layers", 32)),
        }
        self._worker = None
        self._scheduler = None
        if role == KVConnectorRole.SCHEDULER:
            self._scheduler = OrchKvConnectorScheduler(orchkv_cfg)
        elif role == KVConnectorRole.WORKER:
            self._worker = OrchKvConnectorWorker(orchkv_cfg)

    # worker side
    def register_kv_caches(self, kv_caches: dict[str, torch.Tensor]):
        assert self._worker is not None
        self._worker.register_kv_caches(kv_caches)

    def start_load_kv(self, forward_context, **kwargs: Any) -> None:
        assert self._worker is not None
        meta = self._connector_metadata
        if isinstance(meta, OrchKvConnectorMetadata):
            self._worker.start_load_kv(meta)

    def wait_for_layer_load(self, layer_name: str) -> None:
        assert self._worker is not None
        self._worker.wait_for_layer_load(layer_name)

    def save_kv_layer(self, layer_name: str, kv_layer: torch.Tensor, attn_metadata,
                      **kwargs: Any) -> None:
        assert self._worker is not None
        meta = self._connector_metadata
        if isinstance(meta, OrchKvConnectorMetadata):
            self._worker.save_kv_layer(layer_name, kv_layer, meta)

    def wait_for_save(self):
        assert self._worker is not None
        self._worker.wait_for_save()

    def handle_preemptions(self, preempted_req_ids: set[str]):
        if self._scheduler is not None:
            self._scheduler.handle_preemptions(preempted_req_ids)

    def shutdown(self):
        if self._worker is not None:
            self._worker.shutdown()

    # scheduler side
    def get_num_new_matched_tokens(self, request, num_computed_tokens: int):
        assert self._scheduler is not None
        return self._scheduler.get_num_new_matched_tokens(request, num_computed_tokens)

    def update_state_after_alloc(self, request, blocks, num_external_tokens: int):
        assert self._scheduler is not None
        self._scheduler.update_state_after_alloc(request, blocks, num_external_tokens)

    def build_connector_meta(self, scheduler_output):
        assert self._scheduler is not None
        return self._scheduler.build_connector_meta(scheduler_output)

    def request_finished(self, request, block_ids: list[int]):
        assert self._scheduler is not None
        return self._scheduler.request_finished(request, block_ids)
