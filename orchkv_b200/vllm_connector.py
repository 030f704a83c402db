"""vLLM V1 KV connector on the B200 path.

The reference's python/orchkv/vllm_integration/connector.py with the same
classes, methods, metadata and statistics; the worker's data plane is
batched: a layer's save is one copy launch gathering every listed block of
the layer's cache tensor into a pinned store, a layer's load one launch
scattering them back (the reference: one ``copy_`` per block and layer,
connector.py:136-195).  The scheduler side keeps one table of the blocks
each finished request left in the store and gives the reference's answers
(connector.py:220-282), pinned by a recorded run of the reference connector.

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
    """Scheduler role: one table, request id -> the blocks that request left
    in the store when it finished, serves both questions the scheduler asks.
    A returning request can reuse as many tokens as the table holds blocks
    for it beyond what is already computed; a preempted request has its
    blocks queued for saving on every layer.  The queues go to the workers in
    the step's metadata and start empty again (the reference's observable
    behaviour, connector.py:227-289)."""

    def __init__(self, orchkv_cfg: dict[str, Any]):
        n_layers = int(orchkv_cfg.get("n_layers", 32))
        self._layer_names = tuple(f"layer_{i}" for i in range(n_layers))
        self._stored: dict[str, set[int]] = {}
        self._save_queue: dict[str, list[int]] = {}
        self._load_queue: dict[str, list[int]] = {}

    def get_num_new_matched_tokens(self, request, num_computed_tokens: int):
        stored = self._stored.get(request.request_id, ())
        reusable = len(stored) - num_computed_tokens
        return (reusable, True) if reusable > 0 else (0, False)

    def update_state_after_alloc(self, request, blocks, num_external_tokens: int):
        """Nothing to record: loads are driven by the table alone."""

    def request_finished(self, request, block_ids: list[int]):
        self._stored[request.request_id] = set(block_ids)
        return False, None

    def handle_preemptions(self, preempted_req_ids: set[str]):
        for rid in preempted_req_ids:
            blocks = self._stored.get(rid)
            if not blocks:
                continue
            for name in self._layer_names:
                self._save_queue.setdefault(name, []).extend(blocks)

    def build_connector_meta(self, scheduler_output) -> OrchKvConnectorMetadata:
        meta = OrchKvConnectorMetadata(blocks_to_save=self._save_queue,
                                       blocks_to_load=self._load_queue)
        self._save_queue, self._load_queue = {}, {}
        return meta


def _connector_settings(vllm_config) -> dict[str, Any]:
    """The data-plane settings of the connector: the connector's extra config
    (dram_pool_gb, tokens_per_block, num_cuda_streams, io_workers, and d_head
    / n_layers where the model config has none), with the model config's
    head_dim and num_layers taking precedence (connector.py:311-331)."""
    ktc = getattr(vllm_config, "kv_transfer_config", None)
    extra = (getattr(ktc, "kv_connector_extra_config", None) or {}) if ktc is not None else {}
    model = getattr(vllm_config, "model_config", None)
    return {
        "dram_pool_bytes": int(extra.get("dram_pool_gb", 8)) << 30,
        "d_head": getattr(model, "head_dim", extra.get("d_head", 128)),
        "tokens_per_block": extra.get("tokens_per_block", 16),
        "num_cuda_streams": extra.get("num_cuda_streams", 4),
        "io_workers": extra.get("io_workers", 4),
        "n_layers": getattr(model, "num_layers", extra.get("n_layers", 32)),
    }


class OrchKvOffloadingConnector(KVConnectorBase_V1):
    """vLLM V1 connector offloading KV blocks through the B200 data plane.
    One object per role: the scheduler role answers prefix-match queries and
    builds the per-step metadata, the worker role moves blocks; each call is
    routed to the role object that serves it (connector.py:285-421)."""

    @property
    def prefer_cross_layer_blocks(self) -> bool:
        return True

    def __init__(self, vllm_config, role, kv_cache_config=None):
        super().__init__(vllm_config, role, kv_cache_config)
        settings = _connector_settings(vllm_config)
        self._scheduler = (OrchKvConnectorScheduler(settings)
                           if role == KVConnectorRole.SCHEDULER else None)
        self._worker = (OrchKvConnectorWorker(settings)
                        if role == KVConnectorRole.WORKER else None)

    def _as_worker(self) -> "OrchKvConnectorWorker":
        if self._worker is None:
            raise RuntimeError("worker call on a connector built for the scheduler role")
        return self._worker

    def _as_scheduler(self) -> OrchKvConnectorScheduler:
        if self._scheduler is None:
            raise RuntimeError("scheduler call on a connector built for the worker role")
        return self._scheduler

    def _step_meta(self):
        meta = self._connector_metadata
        return meta if isinstance(meta, OrchKvConnectorMetadata) else None

    # ---- worker role ----
    def register_kv_caches(self, kv_caches: dict[str, torch.Tensor]):
        self._as_worker().register_kv_caches(kv_caches)

    def start_load_kv(self, forward_context, **kwargs: Any) -> None:
        worker, meta = self._as_worker(), self._step_meta()
        if meta is not None:
            worker.start_load_kv(meta)

    def wait_for_layer_load(self, layer_name: str) -> None:
        self._as_worker().wait_for_layer_load(layer_name)

    def save_kv_layer(self, layer_name: str, kv_layer: torch.Tensor, attn_metadata,
                      **kwargs: Any) -> None:
        worker, meta = self._as_worker(), self._step_meta()
        if meta is not None:
            worker.save_kv_layer(layer_name, kv_layer, meta)

    def wait_for_save(self):
        self._as_worker().wait_for_save()

    def shutdown(self):
        if self._worker is not None:
            self._worker.shutdown()

    # ---- scheduler role ----
    def handle_preemptions(self, preempted_req_ids: set[str]):
        if self._scheduler is not None:
            self._scheduler.handle_preemptions(preempted_req_ids)

    def get_num_new_matched_tokens(self, request, num_computed_tokens: int):
        return self._as_scheduler().get_num_new_matched_tokens(request, num_computed_tokens)

    def update_state_after_alloc(self, request, blocks, num_external_tokens: int):
        self._as_scheduler().update_state_after_alloc(request, blocks, num_external_tokens)

    def build_connector_meta(self, scheduler_output):
        return self._as_scheduler().build_connector_meta(scheduler_output)

    def request_finished(self, request, block_ids: list[int]):
        return self._as_scheduler().request_finished(request, block_ids)
