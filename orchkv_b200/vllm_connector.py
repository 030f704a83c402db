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


class _SlotStore:
    """Pinned copies of one layer's saved blocks, one fixed-size slot per
    block id.  Freed slots are handed out again before the store grows; a
    growth doubles the slot count (16 at least) and is planned, with its
    byte cost, before any slot is assigned."""

    def __init__(self, slot_elems: int, dtype: torch.dtype):
        self.slot_elems, self.dtype = slot_elems, dtype
        self.buf: torch.Tensor | None = None    # [capacity, slot_elems], pinned
        self.where: dict[int, int] = {}         # block id -> slot
        self.spare: list[int] = []              # freed slots
        self.top = 0                            # slots ever handed out

    @property
    def capacity(self) -> int:
        return 0 if self.buf is None else self.buf.shape[0]

    @property
    def slot_bytes(self) -> int:
        return self.slot_elems * self.dtype.itemsize

    def growth_for(self, block_ids: list[int]) -> int:
        """Slot count the store needs to take `block_ids` (its capacity if none)."""
        fresh = len({b for b in block_ids if b not in self.where})
        top = self.top + max(0, fresh - len(self.spare))
        return self.capacity if top <= self.capacity else max(top, 2 * self.capacity, 16)

    def assign(self, block_ids: list[int], capacity: int, busy_streams) -> list[int]:
        """Slots of `block_ids`, new ones assigned, the store grown to
        `capacity` first (copies in flight on the old buffer end before it
        is copied over)."""
        if capacity > self.capacity:
            grown = torch.empty(capacity, self.slot_elems, dtype=self.dtype).pin_memory()
            if self.buf is not None:
                for stream in busy_streams:
                    stream.synchronize()
                grown[: self.buf.shape[0]].copy_(self.buf)
            self.buf = grown
        slots = []
        for b in block_ids:
            if b not in self.where:
                if self.spare:
                    self.where[b] = self.spare.pop()
                else:
                    self.where[b] = self.top
                    self.top += 1
            slots.append(self.where[b])
        return slots

    def drop(self, block_id: int):
        slot = self.where.pop(block_id, None)
        if slot is not None:
            self.spare.append(slot)


class _CopyLane:
    """One copy direction: its CUDA stream and the blocks it was asked to move."""

    def __init__(self):
        self.stream = torch.cuda.Stream()
        self.requested = 0


class OrchKvConnectorWorker:
    """Worker role.  Each layer's saved blocks sit in a pinned slot store; a
    layer's save or load is one orchkv_copy_token_blocks launch between
    vLLM's cache tensor and that store (per-block copies for a cache whose
    blocks are not contiguous chunks), saves on one lane and loads on the
    other, loads ordered after the saves issued before them, and a layer's
    load awaited through the event recorded after it.  The reference worker
    also opens the orchkv data plane with a DRAM pool of `dram_pool_bytes`
    it never copies through; these copies need no pool, so the setting caps
    the pinned bytes the stores may hold instead (a save that would pass it
    raises RuntimeError and changes nothing)."""

    def __init__(self, orchkv_cfg: dict[str, Any]):
        self._pinned_limit = int(orchkv_cfg.get("dram_pool_bytes", 8 << 30))
        self._caches: dict[str, torch.Tensor] = {}
        self._stores: dict[str, _SlotStore] = {}
        self._saves, self._loads = _CopyLane(), _CopyLane()
        self._load_done: dict[str, torch.cuda.Event] = {}
        self._mu = threading.Lock()
        self._C = core()

    def register_kv_caches(self, kv_caches: dict[str, torch.Tensor]):
        self._caches = kv_caches
        logger.info("OrchKvConnector: registered %d KV cache layers", len(kv_caches))

    def _pinned_bytes(self) -> int:
        return sum(st.capacity * st.slot_bytes for st in self._stores.values())

    def _reserve(self, layer_name: str, kv_layer: torch.Tensor,
                 block_ids: list[int]) -> tuple[_SlotStore, list[int]]:
        with self._mu:
            st = self._stores.get(layer_name)
            if st is None:
                st = self._stores[layer_name] = _SlotStore(kv_layer[0].numel(), kv_layer.dtype)
            capacity = st.growth_for(block_ids)
            extra = (capacity - st.capacity) * st.slot_bytes
            if extra and self._pinned_bytes() + extra > self._pinned_limit:
                raise RuntimeError(
                    f"OrchKv: saving {len(block_ids)} blocks of {layer_name} would hold "
                    f"{self._pinned_bytes() + extra} pinned bytes, over dram_pool_bytes "
                    f"({self._pinned_limit})")
            return st, st.assign(block_ids, capacity, (self._saves.stream, self._loads.stream))

    @staticmethod
    def _contiguous_blocks(kv_layer: torch.Tensor) -> bool:
        chunk = kv_layer[0].numel() * kv_layer.element_size()
        return (kv_layer[0].is_contiguous() and kv_layer.stride(0) == kv_layer[0].numel()
                and chunk % 16 == 0 and kv_layer.data_ptr() % 16 == 0)

    def _move(self, kv_layer: torch.Tensor, st: _SlotStore, block_ids: list[int],
              slots: list[int], to_store: bool, stream: torch.cuda.Stream):
        """Blocks between the cache tensor and their slots, on `stream` (the
        caller's current stream)."""
        if not self._contiguous_blocks(kv_layer):
            for b, s in zip(block_ids, slots):
                if to_store:
                    st.buf[s].view(kv_layer[b].shape).copy_(kv_layer[b], non_blocking=True)
                else:
                    kv_layer[b].copy_(st.buf[s].view(kv_layer[b].shape), non_blocking=True)
            return
        dev = kv_layer.device
        ids = torch.tensor(block_ids, dtype=torch.int32).pin_memory().to(dev, non_blocking=True)
        sl = torch.tensor(slots, dtype=torch.int32).pin_memory().to(dev, non_blocking=True)
        chunk = kv_layer[0].numel() * kv_layer.element_size()
        rc = self._C.copy_token_blocks([kv_layer.data_ptr()], 1, 0, chunk, 1, kv_layer.shape[0],
                                       ids.data_ptr(), len(block_ids), st.buf.data_ptr(),
                                       0 if to_store else 1, stream.cuda_stream, sl.data_ptr())
        if rc != 0:
            raise RuntimeError(f"orchkv_copy_token_blocks failed: {rc}")
        ids.record_stream(stream)              # the index tensors live until the copy ran
        sl.record_stream(stream)

    def save_kv_layer(self, layer_name: str, kv_layer: torch.Tensor,
                      metadata: OrchKvConnectorMetadata, block_ids: list[int] | None = None):
        """The listed blocks (the metadata's for this layer by default) into
        the layer's store, asynchronously, after the work already queued on
        the current stream."""
        ids = metadata.blocks_to_save.get(layer_name, []) if block_ids is None else block_ids
        if not ids:
            return
        st, slots = self._reserve(layer_name, kv_layer, ids)
        lane = self._saves
        lane.stream.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(lane.stream):
            self._move(kv_layer, st, ids, slots, True, lane.stream)
        lane.requested += len(ids)

    def wait_for_save(self):
        self._saves.stream.synchronize()

    def start_load_kv(self, metadata: OrchKvConnectorMetadata):
        """Every layer's stored blocks back into the cache tensors,
        asynchronously; blocks with no stored copy are left alone (warned)."""
        lane = self._loads
        lane.stream.wait_stream(torch.cuda.current_stream())
        lane.stream.wait_stream(self._saves.stream)
        for layer_name, ids in metadata.blocks_to_load.items():
            kv_layer = self._caches.get(layer_name)
            if kv_layer is None:
                continue
            with self._mu:
                st = self._stores.get(layer_name)
                held = {b: st.where[b] for b in ids if b in st.where} if st else {}
            for b in ids:
                if b not in held:
                    logger.warning("OrchKv: no DRAM buffer for %s block %d", layer_name, b)
            with torch.cuda.stream(lane.stream):
                if held:
                    self._move(kv_layer, st, list(held), list(held.values()), False,
                               lane.stream)
                self._load_done[layer_name] = lane.stream.record_event()
        lane.requested += sum(len(ids) for ids in metadata.blocks_to_load.values())

    def wait_for_layer_load(self, layer_name: str):
        done = self._load_done.pop(layer_name, None)
        if done is not None:
            done.synchronize()

    def free_blocks(self, layer_name: str, block_ids: list[int]):
        """The stored copies of freed blocks are dropped (their slots reused)."""
        with self._mu:
            st = self._stores.get(layer_name)
            for b in block_ids if st else ():
                st.drop(b)

    def get_stats(self) -> dict[str, Any]:
        with self._mu:
            held = sum(len(st.where) for st in self._stores.values())
        return {"save_count": self._saves.requested, "load_count": self._loads.requested,
                "dram_buffers": held}

    def shutdown(self):
        for lane in (self._saves, self._loads):
            lane.stream.synchronize()
        with self._mu:
            self._stores.clear()


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
