#!/usr/bin/env python
"""Decode-step schedule + migrate benchmark for orchkv_b200 on B200.

Workload (per GPU; weak scaling across ranks): the Qwen2.5-7B-shaped GQA batch
— 32 requests x 8192-token context, 28 layers, 28 query heads, 4 KV heads,
d_head 128, bf16 KV, 16-token blocks (8 KiB slabs, 1,835,008 slabs, 14 GiB).
Synthetic, seeded inputs: attention logits N(0, 2) with 1% heavy-hitter
tokens +6 per (row, head), softmaxed over the context; KV values N(0, 1).

Steady state: 5% of the blocks (the coldest when the run starts) sit in the
pinned DRAM tier, evicted in an earlier step; the other 95% are in HBM.

One step (everything resident in HBM when it starts):
  append 1 token per (request, layer)       -> paged append kernel
  per-block attention mass, EMA, hotness    -> scoring + step/classify sweep
  coldest 25% of all blocks among those in HBM -> radix select
  5% prefetch set (top EMA among DRAM)      -> radix select
  evict the first set to DRAM and promote   -> one swap: pack + copy engine
  the second, at once                          D2H, copy engine H2D + unpack
  read the step's result counts back to the host.
Between timed steps (not timed) the step's victims are promoted back and the
prefetch set evicted again, so every step starts from the same state.

value = migrated blocks (evicted + promoted) per second, whole job.
e2e   = the same step through the C ABI with host inputs: attention
        probabilities and new tokens copied from pinned host memory inside
        the timed region.
--impl reference times the reference's own C scheduler and per-block
migration path (compiled from its sources into oracle/_ref) on a sample of
the requests, one request per host thread.
"""
from __future__ import annotations

import argparse
import ctypes as C
import json
import os
import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "decode-step schedule+migrate µs and migrated blocks/s per GPU; HBM GB/s % peak"
WL = dict(name="qwen2.5-7b-gqa-decode-step", B=32, L=28, Hq=28, Hkv=4, D=128, T=8192, tpb=16)
EVICT_FRAC, PROMOTE_FRAC = 0.25, 0.05
# DRAM bytes (read + write) of one score launch per request of this workload:
# 216.95 MB measured by ncu (dram__bytes_read.sum + dram__bytes_write.sum) on one
# 8-request launch; the launch streams each request's rows once, so it scales
SCORE_TRAFFIC_PER_REQUEST = 216.95e6 / 8
# DRAM bytes (read + write) of one pack launch over a full staging chunk of
# 32,768 slabs (536.9 MB of algorithmic bytes): 268.58 MB read + 216.66 MB
# written by ncu on an 8-request step (the rest of its writes are still in L2
# when the launch ends)
PACK_TRAFFIC_PER_FULL_LAUNCH = 268.58e6 + 216.66e6
PACK_FULL_LAUNCH_BYTES = 2 * 32768 * 8192
NOMINAL_HBM_GBS = 7700.0          # B200 HBM3e, HGX figure


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as fh:
            p = json.load(fh)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi clock/throttle samples while the timed region runs."""

    def __init__(self, index):
        self.index = index
        self.rows = []
        self.proc = None

    def __enter__(self):
        q = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
             "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
             "clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), "--query-gpu=" + q,
                 "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            parts = [x.strip() for x in line.split(",")]
            if len(parts) == 7:
                self.rows.append(parts)

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[0]) for r in self.rows if r[0].replace(".", "").isdigit()]
        mx = [float(r[1]) for r in self.rows if r[1].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in self.rows for i in range(4) if r[3 + i] == "Active"})
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(mx) if mx else None, "reasons": reasons,
                "samples": len(self.rows)}


# ---------------------------------------------------------------------------
# B200 arm
# ---------------------------------------------------------------------------

class Workload:
    """The decode-step workload on this rank.  staging: "whole" sizes the
    evict staging buffer to a whole step's evict (what lets the swap overlap
    both copy directions); "ring" keeps the library's default 3-slot ring, so
    a step's 14 chunks reuse slots."""

    def __init__(self, torch, okv, rank, world, comm=None, seed=0, staging="whole"):
        self.t, self.okv, self.L = torch, okv, okv.lib()
        w = WL
        self.B, self.Ly, self.Hq, self.Hkv, self.D, self.T, self.tpb = (
            w["B"], w["L"], w["Hq"], w["Hkv"], w["D"], w["T"], w["tpb"])
        self.nb = self.T // self.tpb
        self.n_blocks = self.B * self.Ly * self.Hkv * self.nb
        self.slab = self.tpb * self.D * 2 * 2
        self.rows = self.B * self.Ly
        self.k_evict = int(EVICT_FRAC * self.n_blocks)
        self.k_promote = int(PROMOTE_FRAC * self.n_blocks)
        # with a communicator, selections are global: the promote k covers all ranks
        self.k_promote_sel = self.k_promote * world
        self.k_evict_sel = self.k_evict * world
        self.world = world
        torch_ = torch
        dev = torch_.cuda.current_device()
        self.stream = torch_.cuda.current_stream()
        L = self.L
        extra = self.B * self.Ly * self.Hkv * 4           # appended blocks over a run
        cfg = okv.make_config(gpu_pool_bytes=(self.n_blocks + extra + 4096) * self.slab,
                              dram_pool_bytes=(self.k_evict + self.k_promote + 4096) * self.slab,
                              tokens_per_block=self.tpb, d_head=self.D, dtype=1, device=dev,
                              max_blocks_per_head=self.nb + 8)
        ext = okv.OrchkvConfigExt()
        ext.max_blocks = 1 << 21
        # staging for a whole step's evict, so the swap can overlap both directions
        ext.staging_mb = (self.k_evict * self.slab >> 20) + 256 if staging == "whole" else 0
        rc = L.orchkv_init_ext(C.byref(cfg), C.byref(ext))
        if rc != 0:
            raise RuntimeError(f"orchkv_init_ext failed: {rc}")
        L.orchkv_set_stream(C.c_void_p(self.stream.cuda_stream))
        self.tm = okv.Manager(tracker_cap=1 << 21, max_blocks=1 << 22, ema_lambda=0.9,
                              alpha=0.5, beta=0.3, gamma=0.2, recency_tau=50.0)
        assert L.orchkv_attach_scheduler(self.tm.ref) == 0
        assert L.tm_profile_reports(self.tm.ref, 1) == 0      # the score kernel's own time
        if comm:
            assert L.tm_set_comm(self.tm.ref, comm) == 0
        g = torch_.Generator(device="cuda").manual_seed(seed + 1000 * rank)
        self.ctxs = [L.orchkv_request_create(rank * 1000 + i, self.Ly, self.Hkv)
                     for i in range(self.B)]
        assert all(self.ctxs)
        self.arr = (C.c_void_p * self.B)(*self.ctxs)
        for c in self.ctxs:
            for layer in range(self.Ly):
                kv = torch_.randn(2, self.Hkv, self.T, self.D, generator=g, device="cuda",
                                  dtype=torch_.bfloat16)
                assert L.orchkv_prefill(c, layer, kv[0].data_ptr(), kv[1].data_ptr(), self.T) == 0
        # attention probabilities: logits N(0,2), 1% heavy hitters +6, softmax
        probs = torch_.randn(self.rows, self.Hq, self.T, generator=g, device="cuda") * 2.0
        n_hh = max(1, self.T // 100)
        pos = torch_.randint(0, self.T, (self.rows, self.Hq, n_hh), generator=g, device="cuda")
        probs.scatter_add_(2, pos, torch_.full(pos.shape, 6.0, device="cuda"))
        self.probs = torch_.softmax(probs, dim=-1)
        del probs, pos
        self.ids = torch_.empty(self.rows * self.Hkv * self.nb, dtype=torch_.int32, device="cuda")
        self.tok = torch_.randn(2, self.B, self.Ly, self.Hkv, self.D, generator=g, device="cuda",
                                dtype=torch_.bfloat16)
        self.victims = torch_.empty(1 << 21, dtype=torch_.int32, device="cuda")
        self.pref = torch_.empty(1 << 21, dtype=torch_.int32, device="cuda")
        self.reserve = torch_.empty(1 << 21, dtype=torch_.int32, device="cuda")
        # counts words: 0 victims, 1 prefetch set, 2-5 swap {evicted, skipped,
        # promoted, skipped}, 8 restore set, 9-10 restore result, 12 reserve
        # set, 13-14 reserve evict result
        self.counts = torch_.zeros(16, dtype=torch_.int32, device="cuda")
        self.h_counts = torch_.zeros(16, dtype=torch_.int32).pin_memory()
        # host copies for the end-to-end variant
        self.h_probs = self.probs.cpu().pin_memory()
        self.h_tok = self.tok.cpu().pin_memory()
        torch_.cuda.synchronize()
        self.ev = [torch_.cuda.Event(enable_timing=True) for _ in range(10)]
        # the DRAM-resident reserve: one scoring pass, then the coldest 5%
        L, tm = self.L, self.tm.ref
        assert L.orchkv_block_id_table(self.arr, self.B, self.T, self._ptr(self.ids)) == 0
        assert L.tm_report_attn_probs(tm, self._ptr(self.probs), self.rows, self.Hq, self.Hkv,
                                      self.T, self.tpb, None, self._ptr(self.ids)) == 0
        assert L.tm_step_and_classify(tm) == 0
        assert L.tm_select_victims(tm, self.k_promote_sel, self._ptr(self.reserve),
                                   self._ptr(self.counts, 48)) == 0
        self._evict_reserve()
        torch_.cuda.synchronize()

    def _ptr(self, t, off=0):
        return C.c_void_p(t.data_ptr() + off)

    def step(self, e2e=False, check=None):
        """One decode step; returns nothing (results land in self.counts).
        check (tests only, never timed): called with "scored" after the
        scoring launch and with "selected" before the swap."""
        L, t, tm = self.L, self.t, self.tm.ref
        ev = self.ev
        ev[0].record()
        if e2e:
            # host buffers straight into the C ABI: the library copies them in
            probs = self.h_probs
            kp, vp = self.h_tok[0].data_ptr(), self.h_tok[1].data_ptr()
        else:
            probs = self.probs
            kp, vp = self.tok[0].data_ptr(), self.tok[1].data_ptr()
        rc = L.orchkv_append_token_batch(self.arr, self.B, C.c_void_p(kp), C.c_void_p(vp))
        assert rc == 0, rc
        ev[1].record()
        assert L.orchkv_block_id_table(self.arr, self.B, self.T, self._ptr(self.ids)) == 0
        ev[2].record()
        assert L.tm_report_attn_probs(tm, self._ptr(probs), self.rows, self.Hq, self.Hkv,
                                      self.T, self.tpb, None, self._ptr(self.ids)) == 0
        ev[3].record()
        if check:
            check("scored")
        assert L.tm_step_and_classify(tm) == 0
        assert L.tm_select_victims(tm, self.k_evict_sel, self._ptr(self.victims),
                                   self._ptr(self.counts)) == 0
        assert L.tm_select_prefetch(tm, self.k_promote_sel, 0.0, 0.0, self._ptr(self.pref),
                                    self._ptr(self.counts, 4)) == 0
        ev[4].record()
        if check:
            check("selected")
        if e2e:
            # the next step's probabilities start uploading now, on the
            # manager's copy stream, while this step's swap moves blocks; the
            # next step's report reads that copy (one upload per step)
            assert L.tm_stage_input_async(tm, C.c_void_p(self.h_probs.data_ptr()),
                                          self.h_probs.numel() * 4) == 0
        assert L.orchkv_swap_batch(self._ptr(self.victims), self._ptr(self.counts), 1 << 21,
                                   self._ptr(self.pref), self._ptr(self.counts, 4), 1 << 21,
                                   self._ptr(self.counts, 8)) == 0
        ev[5].record()
        self.h_counts.copy_(self.counts, non_blocking=True)
        ev[6].record()

    def _evict_reserve(self):
        assert self.L.orchkv_evict_batch_to_dram(self._ptr(self.reserve),
                                                 self._ptr(self.counts, 48), 1 << 21,
                                                 self._ptr(self.counts, 52)) == 0

    def restore(self):
        """Promote the step's victims back and evict the reserve again (outside
        the timed region)."""
        L, tm = self.L, self.tm.ref
        # every block off the GPU on every rank (selections are global over ranks)
        assert L.tm_select_prefetch(tm, (1 << 21) * self.world, 0.0, 0.0, self._ptr(self.pref),
                                    self._ptr(self.counts, 32)) == 0
        assert L.orchkv_promote_batch_to_gpu(self._ptr(self.pref), self._ptr(self.counts, 32),
                                             1 << 21, self._ptr(self.counts, 36)) == 0
        self._evict_reserve()
        self.t.cuda.synchronize()

    def phases(self):
        e = self.ev
        names = ["append", "id_table", "score", "classify+select", "swap", "readback"]
        return {n: e[i].elapsed_time(e[i + 1]) for i, n in enumerate(names)}

    def close(self):
        L = self.L
        for c in self.ctxs:
            L.orchkv_request_destroy(c)
        self.tm.close()
        L.orchkv_shutdown()


# ---------------------------------------------------------------------------
# Llama-3-8B-shaped pool sharded by KV head (one fixed total pool at every N)
# ---------------------------------------------------------------------------

SH = dict(name="llama-3-8b-kv-head-sharded-capacity-40pct", B=8, L=32, Hq=32, Hkv=8, D=128,
          T=32768, tpb=64, capacity=0.4, zipf=1.1)


def orderable_u32(x):
    """Ascending uint32 key of ascending float32 values (-0 as +0, NaN last),
    the selection's key order."""
    x = np.asarray(x, np.float32).copy()
    x[x == 0.0] = 0.0
    u = x.view(np.uint32)
    k = np.where(u & np.uint32(0x80000000), ~u, u | np.uint32(0x80000000)).astype(np.uint32)
    k[np.isnan(x)] = 0xFFFFFFFE
    return k


class ShardedWorkload:
    """The Llama-3-8B-shaped pool (32 layers, 32 query / 8 KV heads, d_head
    128, fp16, 64-token blocks, 32,768-token context) with its KV heads split
    over the ranks: rank r holds KV heads [r*8/N, (r+1)*8/N) of every request
    and the attention probabilities of their query heads, so the total pool
    is the same at every N.  Probabilities: per (request, layer, KV head) a
    Zipf(1.1) block mass over the blocks in a seeded order, spread over each
    block's tokens with a seeded +-50% per-token jitter, normalised per query
    head -- drawn per global KV head, so every N sees the same numbers.
    A step: append one token per (request, layer), score, classify, select
    the global coldest 60% of all ranks' blocks (GPU capacity 40%; the key
    histograms are all-reduced over NCCL), evict them to the rank's pinned
    DRAM tier, read the counts back.  The restore (untimed) promotes them."""

    def __init__(self, torch, okv, rank, world, comm, requests, seed=0):
        w = SH
        self.t, self.L = torch, okv.lib()
        self.world, self.rank = world, rank
        self.B, self.Ly, self.D, self.T, self.tpb = requests, w["L"], w["D"], w["T"], w["tpb"]
        self.G = w["Hq"] // w["Hkv"]
        self.hkv = w["Hkv"] // world
        self.hq = self.hkv * self.G
        self.nb = self.T // self.tpb
        self.rows = self.B * self.Ly
        self.n_local = self.rows * self.hkv * self.nb
        self.n_total = self.rows * w["Hkv"] * self.nb
        self.slab = self.tpb * self.D * 2 * 2
        self.k_global = self.n_total - int(w["capacity"] * self.n_total)
        extra = self.rows * self.hkv * 4
        cap = 1
        while cap < self.n_local + extra + 1024:
            cap <<= 1
        self.cap = cap
        # a rank's share of the global coldest 60% is 60% of its blocks up to
        # the boundary ties (split in rank order): room for 75% + the appends
        dram = int(0.75 * self.n_local) + extra + 4096
        cfg = okv.make_config(gpu_pool_bytes=(self.n_local + extra + 1024) * self.slab,
                              dram_pool_bytes=dram * self.slab, tokens_per_block=self.tpb,
                              d_head=self.D, dtype=0, device=torch.cuda.current_device(),
                              max_blocks_per_head=self.nb + 8)
        ext = okv.OrchkvConfigExt()
        ext.max_blocks = cap
        L = self.L
        rc = L.orchkv_init_ext(C.byref(cfg), C.byref(ext))
        if rc != 0:
            raise RuntimeError(f"orchkv_init_ext (sharded pool) failed: {rc}")
        self.stream = torch.cuda.current_stream()
        L.orchkv_set_stream(C.c_void_p(self.stream.cuda_stream))
        self.tm = okv.Manager(tracker_cap=cap, max_blocks=2 * cap, ema_lambda=0.9, alpha=0.5,
                              beta=0.3, gamma=0.2, recency_tau=50.0)
        assert L.orchkv_attach_scheduler(self.tm.ref) == 0
        if comm:
            assert L.tm_set_comm(self.tm.ref, comm) == 0
        g = torch.Generator(device="cuda").manual_seed(seed + 7 * rank + 1)
        self.ctxs = [L.orchkv_request_create(i, self.Ly, self.hkv) for i in range(self.B)]
        assert all(self.ctxs)
        self.arr = (C.c_void_p * self.B)(*self.ctxs)
        for c in self.ctxs:
            for layer in range(self.Ly):
                kv = torch.randn(2, self.hkv, self.T, self.D, generator=g, device="cuda",
                                 dtype=torch.float16)
                assert L.orchkv_prefill(c, layer, kv[0].data_ptr(), kv[1].data_ptr(), self.T) == 0
        del kv
        zipf = torch.arange(1, self.nb + 1, dtype=torch.float64, device="cuda") ** -w["zipf"]
        zipf = (zipf / zipf.sum()).float()
        self.probs = torch.empty(self.rows, self.hq, self.T, device="cuda")
        for j in range(self.hkv):
            gh = rank * self.hkv + j                          # global KV head
            gg = torch.Generator(device="cuda").manual_seed(seed * 1000 + 100 + gh)
            order = torch.argsort(torch.rand(self.rows, self.nb, generator=gg, device="cuda"), 1)
            mass = zipf[order]                                # [rows, nb]
            tok = mass.repeat_interleave(self.tpb, dim=1) / self.tpb
            for q in range(self.G):
                jit = 0.5 + torch.rand(self.rows, self.T, generator=gg, device="cuda")
                p = tok * jit
                self.probs[:, j * self.G + q] = p / p.sum(1, keepdim=True)
        del zipf, order, mass, tok, jit, p
        self.ids = torch.empty(self.rows * self.hkv * self.nb, dtype=torch.int32, device="cuda")
        self.tok = torch.randn(2, self.B, self.Ly, self.hkv, self.D, generator=g, device="cuda",
                               dtype=torch.float16)
        self.victims = torch.empty(cap, dtype=torch.int32, device="cuda")
        self.pref = torch.empty(cap, dtype=torch.int32, device="cuda")
        self.counts = torch.zeros(16, dtype=torch.int32, device="cuda")
        self.h_counts = torch.zeros(16, dtype=torch.int32).pin_memory()
        self.ev = [torch.cuda.Event(enable_timing=True) for _ in range(7)]
        torch.cuda.synchronize()

    def _ptr(self, t, off=0):
        return C.c_void_p(t.data_ptr() + off)

    def step(self, check=None):
        L, tm, ev = self.L, self.tm.ref, self.ev
        ev[0].record()
        assert L.orchkv_append_token_batch(self.arr, self.B, self._ptr(self.tok[0]),
                                           self._ptr(self.tok[1])) == 0
        ev[1].record()
        assert L.orchkv_block_id_table(self.arr, self.B, self.T, self._ptr(self.ids)) == 0
        ev[2].record()
        assert L.tm_report_attn_probs(tm, self._ptr(self.probs), self.rows, self.hq, self.hkv,
                                      self.T, self.tpb, None, self._ptr(self.ids)) == 0
        ev[3].record()
        assert L.tm_step_and_classify(tm) == 0
        assert L.tm_select_victims(tm, self.k_global, self._ptr(self.victims),
                                   self._ptr(self.counts)) == 0
        ev[4].record()
        if check:
            check()
        # counts words: 0 picks, 2-3 evict {evicted, skipped}, 8 restore set,
        # 9-10 restore {promoted, skipped}; _ptr offsets are in bytes
        assert L.orchkv_evict_batch_to_dram(self._ptr(self.victims), self._ptr(self.counts),
                                            self.cap, self._ptr(self.counts, 8)) == 0
        ev[5].record()
        self.h_counts.copy_(self.counts, non_blocking=True)
        ev[6].record()

    def restore(self):
        """Every evicted block back to HBM (untimed; the prefetch selection is
        global too, so every rank takes the same collective steps)."""
        L, tm = self.L, self.tm.ref
        assert L.tm_select_prefetch(tm, self.cap * self.world, 0.0, 0.0, self._ptr(self.pref),
                                    self._ptr(self.counts, 32)) == 0
        assert L.orchkv_promote_batch_to_gpu(self._ptr(self.pref), self._ptr(self.counts, 32),
                                             self.cap, self._ptr(self.counts, 36)) == 0
        self.t.cuda.synchronize()

    def phases(self):
        e = self.ev
        names = ["append", "id_table", "score", "classify+select", "evict", "readback"]
        return {n: e[i].elapsed_time(e[i + 1]) for i, n in enumerate(names)}

    def selection_view(self):
        """This rank's hotness, eligibility (tracker and classifier active, in
        HBM, not migrating) and picks, for the global coldest-k check."""
        st = self.tm.state()
        loc = np.zeros(self.cap, np.uint32)
        state = np.zeros(self.cap, np.uint8)
        assert self.L.orchkv_read_block_locs(loc.ctypes.data, state.ctypes.data) == 0
        elig = (st["t_active"] & st["c_active"] & ((loc >> 29) == 0) & (state != 5)).astype(bool)
        n = int(self.counts[0].item())
        picks = self.victims[:n].cpu().numpy().view(np.uint32).astype(np.int64)
        return st["hot"], elig, picks

    def close(self):
        L = self.L
        for c in self.ctxs:
            L.orchkv_request_destroy(c)
        self.tm.close()
        L.orchkv_shutdown()


def run_sharded(args, torch, okv, rank, world, comm, dist, link_d2h):
    """The KV-head-sharded pool: K timed steps (W warm-up), each bracketed by
    a barrier and a synchronize, step time = max over ranks; then one checked
    step whose global picks are compared (rank 0) with a stable (hotness,
    rank, slot) sort of all ranks' eligible blocks.  Returns the line's
    `sharded` object on rank 0."""
    if SH["Hkv"] % world:
        return {"skipped": f"{SH['Hkv']} KV heads do not split over {world} ranks"}

    def barrier():
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    sw = ShardedWorkload(torch, okv, rank, world, comm, args.sharded_requests)
    L = sw.L
    for _ in range(max(1, min(args.warmup, 2))):
        sw.step()
        sw.restore()
    if comm:
        L.orchkv_comm_exchange_time(comm, C.byref(C.c_float()), C.byref(C.c_uint32()))
    step_ms, ph_acc, evicted, xch = [], {}, 0, [0.0, 0]
    n_steps = min(args.steps, 5)          # a secondary workload: a few steps keep the run short
    pk_ms, pk_bytes, pk_chunks, pr_ms = C.c_float(), C.c_ulonglong(), C.c_uint32(), C.c_float()
    chunk_ms, n_chunk_ms = (C.c_float * 1024)(), C.c_uint32()
    for i in range(n_steps):
        barrier()
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0.record()
        sw.step()
        t1.record()
        barrier()
        step_ms.append(t0.elapsed_time(t1))
        for k, v in sw.phases().items():
            ph_acc.setdefault(k, []).append(v)
        evicted += sw.h_counts.tolist()[2]            # the evict's {evicted, skipped}: words 2-3
        if comm:
            ms, calls = C.c_float(), C.c_uint32()
            L.orchkv_comm_exchange_time(comm, C.byref(ms), C.byref(calls))
            xch[0] += ms.value
            xch[1] += calls.value
        if i == n_steps - 1:                          # the last timed evict's pack kernels
            L.orchkv_last_migration_profile(C.byref(pk_ms), C.byref(pk_bytes),
                                            C.byref(pk_chunks), C.byref(pr_ms))
            L.orchkv_last_pack_chunks(chunk_ms, 1024, C.byref(n_chunk_ms))
        sw.restore()
    chunk_ms = [chunk_ms[i] for i in range(min(1024, n_chunk_ms.value))]
    hbm_peak = peaks()[0]
    # checked step (untimed): the ranks' union of picks vs the global order
    view = {}
    sw.step(check=lambda: view.update(v=sw.selection_view()))
    sw.restore()
    hot, elig, picks = view["v"]
    if world > 1:
        parts = [None] * world
        dist.all_gather_object(parts, (hot, elig, picks))
    else:
        parts = [(hot, elig, picks)]
    phases = {k: sum(v) / len(v) for k, v in ph_acc.items()}
    mean_ms = sum(step_ms) / len(step_ms)
    ev_ms = phases["evict"]
    d2h = evicted / n_steps * sw.slab / (ev_ms * 1e-3) / 1e9
    t = torch.tensor([mean_ms, evicted / n_steps, d2h, xch[0] / n_steps, link_d2h],
                     dtype=torch.float64, device="cuda")
    if world > 1:
        allv = [torch.zeros_like(t) for _ in range(world)]
        dist.all_gather(allv, t)
        allv = [x.tolist() for x in allv]
    else:
        allv = [t.tolist()]
    out = None
    if rank == 0:
        hot_all = np.concatenate([p[0] for p in parts])
        elig_all = np.concatenate([p[1] for p in parts])
        got = np.sort(np.concatenate([p[2] + r * sw.cap for r, p in enumerate(parts)]))
        idx = np.nonzero(elig_all)[0]
        order = np.lexsort((idx, orderable_u32(hot_all[idx])))[:sw.k_global]
        want = np.sort(idx[order])
        parity = bool(len(got) == len(want) == sw.k_global and np.array_equal(got, want))
        ms_max = max(r[0] for r in allv)
        moved = sum(r[1] for r in allv)
        out = {
            "workload": SH["name"], "requests": sw.B, "context": sw.T, "layers": sw.Ly,
            "q_heads": SH["Hq"], "kv_heads": SH["Hkv"], "kv_heads_per_gpu": sw.hkv,
            "d_head": sw.D, "tokens_per_block": sw.tpb, "dtype": "fp16",
            "blocks_total": sw.n_total, "blocks_per_gpu": sw.n_local,
            "pool_gib_total": round(sw.n_total * sw.slab / 2**30, 2),
            "gpu_capacity": SH["capacity"], "evict_per_step_total": sw.k_global,
            "sample": f"{sw.B} of the configuration's 64 requests (host RAM for the pinned "
                      f"DRAM tier at every N); the same {sw.B} requests at every N",
            "steps": n_steps, "ms_per_step": round(ms_max, 3),
            "value": round(moved / (ms_max * 1e-3), 1), "unit": "evicted blocks/s (all ranks)",
            "scaling": "strong (fixed total pool)",
            "per_rank_evict_d2h_gbs": [round(r[2], 1) for r in allv],
            "summed_evict_d2h_gbs": round(sum(r[2] for r in allv), 1),
            "probe_d2h_gbs_per_rank": [round(r[4], 1) for r in allv],
            "probe_d2h_gbs_summed": round(sum(r[4] for r in allv), 1),
            "collective_ms_per_step": [round(r[3], 4) for r in allv] if world > 1 else None,
            "phases_ms_rank0": {k: round(v, 4) for k, v in phases.items()},
            "pack_rank0": {"kernel": "evict pack (HBM gather -> staging ring), 32 KB slabs",
                           "ms": round(pk_ms.value, 4), "bytes": pk_bytes.value,
                           "achieved_gbs": round(pk_bytes.value / max(pk_ms.value, 1e-9) / 1e6, 1),
                           "frac": round(pk_bytes.value / max(pk_ms.value, 1e-9) / 1e6
                                         / hbm_peak, 4),
                           "first_chunk": pack_first_chunk(chunk_ms, pk_bytes.value,
                                                           pk_chunks.value, hbm_peak),
                           "chunks": pk_chunks.value},
            "limiter": {
                "phase": "evict (gather-pack + device-to-host drain)",
                "share_of_step_rank0": round(ev_ms / mean_ms, 3),
                "frac_of_d2h_probe_per_rank": [round(r[2] / r[4], 3) if r[4] else None
                                               for r in allv],
                "bound": f"the box's host link, device-to-host: {sum(r[4] for r in allv):.1f} "
                         f"GB/s summed over {world} rank(s), probed with all ranks copying"},
            "parity": {"global_coldest_k_equal": parity, "checked_blocks": int(len(idx)),
                       "rule": "union of the ranks' picks == the k smallest (hotness, rank, "
                               "slot) over every rank's eligible blocks"},
        }
    sw.close()
    if out is not None and world == 1 and not args.no_cpu_baseline:
        out["cpu_baseline"] = _ref_pool_sample((SH["L"], SH["Hq"], SH["Hkv"], SH["D"], SH["T"],
                                                SH["tpb"]), 0, 1.0 - SH["capacity"])
    return out


# ---------------------------------------------------------------------------
# Mistral-7B-shaped time-multiplexed pool, KV heads sharded over the ranks
# ---------------------------------------------------------------------------

MX = dict(name="mistral-7b-time-multiplexed-4-sub-batches", B=32, L=32, Hq=32, Hkv=8, D=128,
          T=4096, tpb=16, sub_batches=4, resident=2)


class MultiplexedWorkload:
    """The Mistral-7B-shaped shared pool (32 layers, 32 query / 8 KV heads,
    d_head 128, bf16, 16-token blocks, 4096-token context) rotated through
    the GPU in four sub-batches of requests, two resident at a time, KV heads
    split over the ranks like the sharded pool.  A step scores the resident
    sub-batches' query rows (logits N(0, 1.5), softmax), classifies, and one
    orchkv_swap_batch evicts the older resident sub-batch while promoting the
    next one from the DRAM tier: half of the GPU's blocks leave and half
    arrive, every step, with no restore between steps."""

    def __init__(self, torch, okv, rank, world, requests, seed=0):
        w = MX
        self.t, self.L = torch, okv.lib()
        self.B, self.Ly, self.D, self.T, self.tpb = requests, w["L"], w["D"], w["T"], w["tpb"]
        self.S = w["sub_batches"]
        if self.B % self.S:
            raise ValueError("requests must split into the sub-batches")
        self.G = w["Hq"] // w["Hkv"]
        self.hkv = w["Hkv"] // world
        self.hq = self.hkv * self.G
        self.nb = self.T // self.tpb
        self.per_sb = self.B // self.S                          # requests per sub-batch
        self.rows_sb = self.per_sb * self.Ly
        self.blocks_sb = self.rows_sb * self.hkv * self.nb      # this rank's blocks per sub-batch
        self.n_total = self.B * self.Ly * w["Hkv"] * self.nb
        self.slab = self.tpb * self.D * 2 * 2
        cap = 1
        while cap < self.S * self.blocks_sb + 1024:
            cap <<= 1
        self.cap = cap
        resident = w["resident"] * self.blocks_sb
        cfg = okv.make_config(gpu_pool_bytes=(self.S * self.blocks_sb + 1024) * self.slab,
                              dram_pool_bytes=(resident + self.blocks_sb + 1024) * self.slab,
                              tokens_per_block=self.tpb, d_head=self.D, dtype=1,
                              device=torch.cuda.current_device(),
                              max_blocks_per_head=self.nb + 8)
        ext = okv.OrchkvConfigExt()
        ext.max_blocks = cap
        # staging for a whole sub-batch, so each swap overlaps both directions
        ext.staging_mb = (self.blocks_sb * self.slab >> 20) + 256
        L = self.L
        rc = L.orchkv_init_ext(C.byref(cfg), C.byref(ext))
        if rc != 0:
            raise RuntimeError(f"orchkv_init_ext (multiplexed pool) failed: {rc}")
        self.stream = torch.cuda.current_stream()
        L.orchkv_set_stream(C.c_void_p(self.stream.cuda_stream))
        self.tm = okv.Manager(tracker_cap=cap, max_blocks=2 * cap, ema_lambda=0.9, alpha=0.5,
                              beta=0.3, gamma=0.2, recency_tau=50.0)
        assert L.orchkv_attach_scheduler(self.tm.ref) == 0
        g = torch.Generator(device="cuda").manual_seed(seed + 11 * rank + 3)
        self.ctxs = [L.orchkv_request_create(i, self.Ly, self.hkv) for i in range(self.B)]
        assert all(self.ctxs)
        for c in self.ctxs:
            for layer in range(self.Ly):
                kv = torch.randn(2, self.hkv, self.T, self.D, generator=g, device="cuda",
                                 dtype=torch.bfloat16)
                assert L.orchkv_prefill(c, layer, kv[0].data_ptr(), kv[1].data_ptr(), self.T) == 0
        del kv
        # per sub-batch: its requests, their block ids ([rows, kv heads, blocks]) and
        # their probabilities, drawn per global KV head so every N sees the same numbers
        self.arrs, self.ids, self.probs = [], [], []
        for sb in range(self.S):
            arr = (C.c_void_p * self.per_sb)(*self.ctxs[sb * self.per_sb:(sb + 1) * self.per_sb])
            ids = torch.empty(self.blocks_sb, dtype=torch.int32, device="cuda")
            assert L.orchkv_block_id_table(arr, self.per_sb, self.T, C.c_void_p(ids.data_ptr())) == 0
            p = torch.empty(self.rows_sb, self.hq, self.T, device="cuda")
            for j in range(self.hkv):
                gg = torch.Generator(device="cuda").manual_seed(seed * 1000 + 500 + 8 * sb +
                                                                rank * self.hkv + j)
                x = torch.randn(self.rows_sb, self.G, self.T, generator=gg, device="cuda") * 1.5
                p[:, j * self.G:(j + 1) * self.G] = torch.softmax(x, -1)
            self.arrs.append(arr)
            self.ids.append(ids)
            self.probs.append(p)
        del x
        self.counts = torch.zeros(16, dtype=torch.int32, device="cuda")
        self.h_counts = torch.zeros(16, dtype=torch.int32).pin_memory()
        self.ev = [torch.cuda.Event(enable_timing=True) for _ in range(5)]
        # start: sub-batches 0 and 1 resident, the others in the DRAM tier
        for sb in range(w["resident"], self.S):
            assert L.orchkv_evict_batch_to_dram(C.c_void_p(self.ids[sb].data_ptr()), None,
                                                self.blocks_sb,
                                                C.c_void_p(self.counts.data_ptr())) == 0
        torch.cuda.synchronize()
        self.t_step = 0

    def checksums(self):
        """Every block's slab checksum, sub-batch by sub-batch (device)."""
        out = []
        for ids in self.ids:
            o = self.t.empty(self.blocks_sb, dtype=self.t.int64, device="cuda")
            assert self.L.orchkv_block_checksums(C.c_void_p(ids.data_ptr()), self.blocks_sb,
                                                 C.c_void_p(o.data_ptr()), None) == 0
            out.append(o)
        assert self.L.orchkv_sync() == 0
        return self.t.cat(out).cpu()

    def step(self):
        L, tm, ev = self.L, self.tm.ref, self.ev
        out_sb = self.t_step % self.S
        in_sb = (self.t_step + MX["resident"]) % self.S
        ev[0].record()
        for sb in (out_sb, (out_sb + 1) % self.S):            # the resident sub-batches
            assert L.tm_report_attn_probs(tm, C.c_void_p(self.probs[sb].data_ptr()),
                                          self.rows_sb, self.hq, self.hkv, self.T, self.tpb,
                                          None, C.c_void_p(self.ids[sb].data_ptr())) == 0
        ev[1].record()
        assert L.tm_step_and_classify(tm) == 0
        ev[2].record()
        assert L.orchkv_swap_batch(C.c_void_p(self.ids[out_sb].data_ptr()), None, self.blocks_sb,
                                   C.c_void_p(self.ids[in_sb].data_ptr()), None, self.blocks_sb,
                                   C.c_void_p(self.counts.data_ptr())) == 0
        ev[3].record()
        self.h_counts.copy_(self.counts, non_blocking=True)
        ev[4].record()
        self.t_step += 1

    def phases(self):
        e = self.ev
        names = ["score", "classify", "swap", "readback"]
        return {n: e[i].elapsed_time(e[i + 1]) for i, n in enumerate(names)}

    def close(self):
        L = self.L
        for c in self.ctxs:
            L.orchkv_request_destroy(c)
        self.tm.close()
        L.orchkv_shutdown()


def run_multiplexed(args, torch, okv, rank, world, dist, link):
    """The time-multiplexed pool: W warm-up steps, K timed steps (barrier +
    synchronize around each, max over ranks), then the rotation completed to
    a multiple of four steps and every block's checksum compared with its
    checksum before the first step (each block has made whole round trips)."""
    if MX["Hkv"] % world:
        return {"skipped": f"{MX['Hkv']} KV heads do not split over {world} ranks"}

    def barrier():
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    mw = MultiplexedWorkload(torch, okv, rank, world, args.multiplexed_requests)
    before = mw.checksums()
    for _ in range(min(args.warmup, 4)):
        mw.step()
    step_ms, ph, moved = [], {}, 0
    n_steps = min(args.steps, 8)          # a secondary workload: two rotations at most
    for _ in range(n_steps):
        barrier()
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0.record()
        mw.step()
        t1.record()
        barrier()
        step_ms.append(t0.elapsed_time(t1))
        for k, v in mw.phases().items():
            ph.setdefault(k, []).append(v)
        c = mw.h_counts.tolist()
        moved += c[0] + c[2]
    ov = [C.c_uint32() for _ in range(3)] + [C.c_int()]
    mw.L.orchkv_last_promote_layout(*[C.byref(x) for x in ov])
    while mw.t_step % MX["sub_batches"]:
        mw.step()
    intact = bool(torch.equal(mw.checksums(), before))
    phases = {k: sum(v) / len(v) for k, v in ph.items()}
    swap_bytes = 2 * mw.blocks_sb * mw.slab
    t = torch.tensor([sum(step_ms) / len(step_ms), moved / n_steps, float(intact),
                      phases["swap"], link["both"]], dtype=torch.float64, device="cuda")
    if world > 1:
        allv = [torch.zeros_like(t) for _ in range(world)]
        dist.all_gather(allv, t)
        allv = [x.tolist() for x in allv]
    else:
        allv = [t.tolist()]
    out = None
    if rank == 0:
        ms_max = max(r[0] for r in allv)
        out = {
            "workload": MX["name"], "requests": mw.B, "context": mw.T, "layers": mw.Ly,
            "q_heads": MX["Hq"], "kv_heads": MX["Hkv"], "kv_heads_per_gpu": mw.hkv,
            "d_head": mw.D, "tokens_per_block": mw.tpb, "dtype": "bf16",
            "sub_batches": MX["sub_batches"], "resident": MX["resident"],
            "blocks_total": mw.n_total, "blocks_per_gpu": mw.S * mw.blocks_sb,
            "pool_gib_total": round(mw.n_total * mw.slab / 2**30, 2),
            "sample": f"{mw.B} of the configuration's 256 requests (host RAM for the DRAM tier "
                      f"at one GPU); the same {mw.B} requests at every N",
            "steps": n_steps, "ms_per_step": round(ms_max, 3),
            "value": round(sum(r[1] for r in allv) / (ms_max * 1e-3), 1),
            "unit": "migrated blocks/s (evicted + promoted, all ranks)",
            "scaling": "strong (fixed total pool)",
            "swap_gbs_per_rank": [round(swap_bytes / (r[3] * 1e-3) / 1e9, 1) for r in allv],
            "probe_both_directions_gbs_per_rank": [round(r[4], 1) for r in allv],
            "swap_overlapped": bool(ov[3].value),
            "phases_ms_rank0": {k: round(v, 4) for k, v in phases.items()},
            "limiter": {
                "phase": "swap (evict and promote, both copy directions at once)",
                "share_of_step_rank0": round(phases["swap"] / (sum(step_ms) / len(step_ms)), 3),
                "frac_of_two_way_probe_per_rank": [
                    round(swap_bytes / (r[3] * 1e-3) / 1e9 / r[4], 3) if r[4] else None
                    for r in allv],
                "bound": f"the box's host link, both directions: "
                         f"{sum(r[4] for r in allv):.1f} GB/s summed over {world} rank(s), "
                         f"probed with all ranks copying"},
            "round_trip_checksums_equal": all(bool(r[2]) for r in allv),
        }
    mw.close()
    if out is not None and world == 1 and not args.no_cpu_baseline:
        out["cpu_baseline"] = _ref_pool_sample((MX["L"], MX["Hq"], MX["Hkv"], MX["D"], MX["T"],
                                                MX["tpb"]), 1, 0.5)
    return out


# ---------------------------------------------------------------------------
# Llama-3-70B-shaped three tiers: HBM 20%, pinned DRAM 50%, files 30%
# ---------------------------------------------------------------------------

TT = dict(name="llama-3-70b-three-tier", B=1, L=80, Hq=64, Hkv=8, D=128, T=131072, tpb=64,
          gpu=0.2, dram=0.5)


class ThreeTierWorkload:
    """The Llama-3-70B-shaped pool over three tiers (80 layers, 64 query / 8
    KV heads, d_head 128, fp16, 64-token blocks, 131,072-token context), KV
    heads split over the ranks.  A step scores (logits N(0, 2), softmax),
    classifies, sends the global coldest 30% two hops to the file tier
    (orchkv_evict_cold_batch: the reference's file layout, 1 MiB runs) and
    the next coldest 50% to pinned DRAM,
    leaving 20% in HBM.  The restore (untimed) promotes the DRAM blocks,
    reads the file blocks back into DRAM and promotes them too."""

    def __init__(self, torch, okv, rank, world, comm, requests, seed=0):
        w = TT
        self.t, self.L = torch, okv.lib()
        self.rank, self.world = rank, world
        self.B, self.Ly, self.D, self.T, self.tpb = requests, w["L"], w["D"], w["T"], w["tpb"]
        self.G = w["Hq"] // w["Hkv"]
        self.hkv = w["Hkv"] // world
        self.hq = self.hkv * self.G
        self.nb = self.T // self.tpb
        self.rows = self.B * self.Ly
        self.n_local = self.rows * self.hkv * self.nb
        self.n_total = self.rows * w["Hkv"] * self.nb
        self.slab = self.tpb * self.D * 2 * 2
        self.k_file = int((1.0 - w["gpu"] - w["dram"]) * self.n_total)
        self.k_dram = int(w["dram"] * self.n_total)
        cap = 1
        while cap < self.n_local + 1024:
            cap <<= 1
        self.cap = cap
        self.base = f"/dev/shm/orchkv_three_tier_r{rank}"
        cfg = okv.make_config(gpu_pool_bytes=(self.n_local + 1024) * self.slab,
                              dram_pool_bytes=(int(0.6 * self.n_local) + 4096) * self.slab,
                              tokens_per_block=self.tpb, d_head=self.D, dtype=0,
                              device=torch.cuda.current_device(),
                              max_blocks_per_head=self.nb + 8)
        cfg.orchfs_base_dir = self.base.encode()
        self.io_workers = max(4, min(16, host_threads()))
        cfg.orchfs_io_workers = self.io_workers
        ext = okv.OrchkvConfigExt()
        ext.max_blocks = cap
        L = self.L
        rc = L.orchkv_init_ext(C.byref(cfg), C.byref(ext))
        if rc != 0:
            raise RuntimeError(f"orchkv_init_ext (three-tier pool) failed: {rc}")
        self.stream = torch.cuda.current_stream()
        L.orchkv_set_stream(C.c_void_p(self.stream.cuda_stream))
        self.tm = okv.Manager(tracker_cap=cap, max_blocks=2 * cap, ema_lambda=0.9, alpha=0.5,
                              beta=0.3, gamma=0.2, recency_tau=50.0)
        assert L.orchkv_attach_scheduler(self.tm.ref) == 0
        if comm:
            assert L.tm_set_comm(self.tm.ref, comm) == 0
        g = torch.Generator(device="cuda").manual_seed(seed + 13 * rank + 5)
        self.ctxs = [L.orchkv_request_create(rank * 1000 + i, self.Ly, self.hkv)
                     for i in range(self.B)]
        assert all(self.ctxs)
        for c in self.ctxs:
            for layer in range(self.Ly):
                kv = torch.randn(2, self.hkv, self.T, self.D, generator=g, device="cuda",
                                 dtype=torch.float16)
                assert L.orchkv_prefill(c, layer, kv[0].data_ptr(), kv[1].data_ptr(), self.T) == 0
        del kv
        self.arr = (C.c_void_p * self.B)(*self.ctxs)
        self.ids = torch.empty(self.n_local, dtype=torch.int32, device="cuda")
        assert L.orchkv_block_id_table(self.arr, self.B, self.T, C.c_void_p(self.ids.data_ptr())) == 0
        # block id -> (request, layer, head, block) for the file tier's lists
        ids_h = self.ids.cpu().numpy().view(np.uint32).astype(np.int64)
        self.where = np.full(cap, -1, np.int64)
        self.where[ids_h] = np.arange(self.n_local)
        self.probs = torch.empty(self.rows, self.hq, self.T, device="cuda")
        for j in range(self.hkv):
            gg = torch.Generator(device="cuda").manual_seed(seed * 1000 + 900 + rank * self.hkv + j)
            for r0 in range(0, self.rows, 16):
                x = torch.randn(min(16, self.rows - r0), self.G, self.T, generator=gg,
                                device="cuda") * 2.0
                self.probs[r0:r0 + 16, j * self.G:(j + 1) * self.G] = torch.softmax(x, -1)
        del x
        self.victims = torch.empty(cap, dtype=torch.int32, device="cuda")
        self.pref = torch.empty(cap, dtype=torch.int32, device="cuda")
        self.counts = torch.zeros(16, dtype=torch.int32, device="cuda")
        self.h_counts = torch.zeros(16, dtype=torch.int32).pin_memory()
        self.files = []                   # per request: the lhb list sent to the file tier
        self.ev = [torch.cuda.Event(enable_timing=True) for _ in range(6)]
        torch.cuda.synchronize()

    def _ptr(self, t, off=0):
        return C.c_void_p(t.data_ptr() + off)

    def _lhb_by_request(self, ids):
        pos = self.where[ids]
        req, rem = np.divmod(pos, self.Ly * self.hkv * self.nb)
        lay, rem = np.divmod(rem, self.hkv * self.nb)
        head, blk = np.divmod(rem, self.nb)
        out = []
        for b in range(self.B):
            m = req == b
            out.append(np.ascontiguousarray(np.stack([lay[m], head[m], blk[m]], 1)
                                            .astype(np.uint32).reshape(-1)))
        return out

    def step(self):
        L, tm, ev = self.L, self.tm.ref, self.ev
        ev[0].record()
        assert L.tm_report_attn_probs(tm, self._ptr(self.probs), self.rows, self.hq, self.hkv,
                                      self.T, self.tpb, None, self._ptr(self.ids)) == 0
        assert L.tm_step_and_classify(tm) == 0
        assert L.tm_select_victims(tm, self.k_file, self._ptr(self.victims),
                                   self._ptr(self.counts)) == 0
        ev[1].record()
        # the coldest 30%: GPU -> (pinned staging) -> the request's file
        n = int(self.counts[0].item())
        vic = self.victims[:n].cpu().numpy().view(np.uint32).astype(np.int64)
        self.files = self._lhb_by_request(vic)
        res = (C.c_uint32 * 2)()
        self.file_moved = 0
        for c, lhb in zip(self.ctxs, self.files):
            if len(lhb):
                assert L.orchkv_evict_cold_batch(c, lhb.ctypes.data, len(lhb) // 3, res) == 0
                self.file_moved += res[0]
        ev[2].record()
        # the next coldest 50%: GPU -> pinned DRAM
        assert L.tm_select_victims(tm, self.k_dram, self._ptr(self.victims),
                                   self._ptr(self.counts)) == 0
        assert L.orchkv_evict_batch_to_dram(self._ptr(self.victims), self._ptr(self.counts),
                                            self.cap, self._ptr(self.counts, 8)) == 0
        ev[3].record()
        self.h_counts.copy_(self.counts, non_blocking=True)
        ev[4].record()

    def restore(self):
        L, tm = self.L, self.tm.ref

        def promote_dram():
            assert L.tm_select_prefetch(tm, self.cap * self.world, 0.0, 0.0, self._ptr(self.pref),
                                        self._ptr(self.counts, 32)) == 0
            assert L.orchkv_promote_batch_to_gpu(self._ptr(self.pref), self._ptr(self.counts, 32),
                                                 self.cap, self._ptr(self.counts, 36)) == 0
        promote_dram()
        res = (C.c_uint32 * 2)()
        for c, lhb in zip(self.ctxs, self.files):
            if len(lhb):
                assert L.orchkv_promote_batch_from_storage(c, lhb.ctypes.data, len(lhb) // 3,
                                                           res) == 0
        promote_dram()
        self.t.cuda.synchronize()

    def checksums(self):
        o = self.t.empty(self.n_local, dtype=self.t.int64, device="cuda")
        tier = self.t.empty(self.n_local, dtype=self.t.uint8, device="cuda")
        assert self.L.orchkv_block_checksums(self._ptr(self.ids), self.n_local, self._ptr(o),
                                             self._ptr(tier)) == 0
        assert self.L.orchkv_sync() == 0
        return o.cpu(), tier.cpu()

    def phases(self):
        e = self.ev
        names = ["score+select", "two-hop to files", "evict to dram", "readback"]
        return {n: e[i].elapsed_time(e[i + 1]) for i, n in enumerate(names)}

    def close(self):
        L = self.L
        for c in self.ctxs:
            L.orchkv_request_destroy(c)
        self.tm.close()
        L.orchkv_shutdown()
        try:
            os.rmdir(self.base)
        except OSError:
            pass


def run_three_tier(args, torch, okv, rank, world, comm, dist):
    """The three-tier pool: W warm-up and K timed steps (wall time with a
    barrier and synchronize around each, as the step's file IO runs on host
    threads; max over ranks), each followed by the untimed restore; every
    block's checksum after the last restore equals its checksum before the
    first step."""
    if TT["Hkv"] % world:
        return {"skipped": f"{TT['Hkv']} KV heads do not split over {world} ranks"}

    def barrier():
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    tw = ThreeTierWorkload(torch, okv, rank, world, comm, args.three_tier_requests)
    before, tier0 = tw.checksums()
    for _ in range(max(1, min(args.warmup, 2))):
        tw.step()
        tw.restore()
    ms, ph, moved_file, moved_dram = [], {}, 0, 0
    n_steps = min(args.steps, 3)          # a secondary workload: seconds per step
    for _ in range(n_steps):
        barrier()
        t0 = time.perf_counter()
        tw.step()
        torch.cuda.synchronize()
        barrier()
        ms.append((time.perf_counter() - t0) * 1e3)
        for k, v in tw.phases().items():
            ph.setdefault(k, []).append(v)
        moved_file += tw.file_moved
        moved_dram += tw.h_counts.tolist()[2]
        tw.restore()
    after, tier1 = tw.checksums()
    intact = bool(torch.equal(before, after) and bool((tier0 == 0).all()) and
                  bool((tier1 == 0).all()))
    phases = {k: sum(v) / len(v) for k, v in ph.items()}
    t = torch.tensor([sum(ms) / len(ms), moved_file / n_steps, moved_dram / n_steps,
                      float(intact), phases["two-hop to files"]], dtype=torch.float64,
                     device="cuda")
    if world > 1:
        allv = [torch.zeros_like(t) for _ in range(world)]
        dist.all_gather(allv, t)
        allv = [x.tolist() for x in allv]
    else:
        allv = [t.tolist()]
    out = None
    if rank == 0:
        ms_max = max(r[0] for r in allv)
        f_tot, d_tot = sum(r[1] for r in allv), sum(r[2] for r in allv)
        out = {
            "workload": TT["name"], "requests": tw.B, "context": tw.T, "layers": tw.Ly,
            "q_heads": TT["Hq"], "kv_heads": TT["Hkv"], "kv_heads_per_gpu": tw.hkv,
            "d_head": tw.D, "tokens_per_block": tw.tpb, "dtype": "fp16",
            "blocks_total": tw.n_total, "pool_gib_total": round(tw.n_total * tw.slab / 2**30, 2),
            "tiers": {"gpu": TT["gpu"], "dram": TT["dram"], "files": round(1 - TT["gpu"] - TT["dram"], 2)},
            "sample": f"{tw.B} of the configuration's 16 requests (host RAM for the pinned DRAM "
                      f"tier and the RAM-backed files at one GPU); the same at every N",
            "file_tier": f"{tw.base} (tmpfs); reads over {tw.io_workers} IO workers",
            "steps": n_steps, "ms_per_step": round(ms_max, 2),
            "value": round((f_tot + d_tot) / (ms_max * 1e-3), 1),
            "unit": "migrated blocks/s (to files + to DRAM, all ranks), wall-timed",
            "scaling": "strong (fixed total pool)",
            "blocks_to_files_per_step": int(f_tot), "blocks_to_dram_per_step": int(d_tot),
            "file_write_gbs_per_rank": [round(r[1] * tw.slab / (r[4] * 1e-3) / 1e9, 2)
                                        for r in allv],
            "phases_ms_rank0": {k: round(v, 3) for k, v in phases.items()},
            "limiter": {
                "phase": "two-hop to files (pack, device-to-host, pwritev)",
                "share_of_step_rank0": round(phases["two-hop to files"] / (sum(ms) / len(ms)), 3),
                "bound": "the file writes: one writer thread per rank copying into the page "
                         "cache (tmpfs)"},
            "round_trip_checksums_equal": all(bool(r[3]) for r in allv),
        }
    tw.close()
    if out is not None and world == 1 and not args.no_cpu_baseline:
        # 8 of the 80 layers: the per-block reference path takes seconds per step
        out["cpu_baseline"] = _ref_pool_sample((8, TT["Hq"], TT["Hkv"], TT["D"], TT["T"],
                                                TT["tpb"]), 0, TT["dram"],
                                               file_frac=1.0 - TT["gpu"] - TT["dram"])
    return out


def _ref_pool_sample(geo, dtype, evict_frac, file_frac=0.0, steps=2):
    """The reference's own path on a one-request sample of a pool's shape
    (its scheduler and per-block data plane compiled from its sources into
    oracle/_ref), on one host core: a step reduces the request's attention
    probabilities (logits N(0, 2), softmax) to per-block mass with the C
    restatement of the managers' reduction, runs the reference scheduler
    (attn_tracker_update_batch, tm_step_done, tm_schedule_once, coldest-first
    order), then sends the coldest `file_frac` of the blocks two hops to its
    file tier (orchkv_evict_cold per block) and the next `evict_frac` to DRAM
    (orchkv_evict_to_dram per block); the restore (untimed) promotes them
    back.  geo = (layers, q heads, kv heads, d_head, tokens, tokens per block).
    Returns migrated blocks/s and the step time."""
    from oracle import oracle as O
    if not O.ref_available():
        return None
    Ly, Hq, Hkv, D, T, tpb = geo
    nb = T // tpb
    n = Ly * Hkv * nb
    slab = tpb * D * 2 * 2
    rng = np.random.default_rng(0)
    probs = np.empty((Ly, Hq, T), np.float32)
    for layer in range(Ly):
        x = rng.normal(0, 2, (Hq, T)).astype(np.float32)
        x = np.exp(x - x.max(-1, keepdims=True))
        probs[layer] = x / x.sum(-1, keepdims=True)
    kv = rng.standard_normal((Hkv, T, D)).astype(np.float16)
    R = O.ref()
    base = b"/dev/shm/orchkv_ref_pool"
    assert R.ref_api_init(0, (n + 64) * slab, (n + 64) * slab, tpb, D, dtype, 4, nb + 8,
                          base) == 0
    ctx = R.ref_api_request_create(0, Ly, Hkv)
    for layer in range(Ly):
        assert R.ref_api_prefill(ctx, layer, kv.ctypes.data, kv.ctypes.data, T) == 0
    rtm = O.RefTM(tracker_cap=n, max_blocks=n, ema_lambda=0.9, alpha=0.5, beta=0.3, gamma=0.2,
                  recency_tau=50.0, cooldown_sec=0.0)
    rtm.register_range(n)
    ids = np.arange(n, dtype=np.uint64)
    k_file, k_all = int(file_frac * n), int((file_frac + evict_frac) * n)
    vict = np.zeros(max(k_all, 1), np.uint64)
    times = []
    for s in range(steps + 1):
        t0 = time.perf_counter()
        mass = O.score_blocks(probs, Hq, Hkv, tpb).reshape(-1)
        c = R.ref_arm_sched_step(rtm.h, ids, mass.copy(), n, 1.0, k_all, vict, np.zeros(3))
        v = vict[:c].astype(np.int64)           # coldest first
        lhb = np.stack([v // (Hkv * nb), (v // nb) % Hkv, v % nb], 1).astype(np.uint32)
        nf = min(k_file, c)
        for i in range(nf):
            assert R.ref_api_evict_cold(ctx, *lhb[i].tolist()) == 0
        rest = np.ascontiguousarray(lhb[nf:].reshape(-1))
        assert R.ref_api_migrate_list(ctx, rest, c - nf, 0, np.zeros(2)) == 0
        dt = time.perf_counter() - t0
        if s:
            times.append(dt)
        for i in range(nf):                      # back to the start (untimed)
            assert R.ref_api_promote_storage(ctx, *lhb[i].tolist()) == 0
        allb = np.ascontiguousarray(lhb.reshape(-1))
        assert R.ref_api_migrate_list(ctx, allb, 0, c, np.zeros(2)) == 0
    R.ref_api_request_destroy(ctx)
    R.ref_api_shutdown()
    rtm.close()
    step_s = statistics.median(times)
    return {"kind": "reference", "cores": 1, "value": round(c / step_s, 1),
            "unit": "migrated blocks/s", "ms_per_step": round(step_s * 1e3, 1),
            "sample": f"1 request x {Ly} layers x {Hkv} KV heads x {nb} blocks ({n} blocks): "
                      f"scheduler step, coldest {round(100 * (file_frac + evict_frac))}% moved "
                      f"block by block; median of {steps} steps after one"}


# ---------------------------------------------------------------------------
# The CPU-runnable scheduler step (one request) as a latency figure
# ---------------------------------------------------------------------------

C1 = dict(name="cpu-runnable-step-1req-8L-4kvh-4096", L=8, Hq=28, Hkv=4, D=128, T=4096, tpb=64,
          hist=16, evict_frac=0.5)


def _c1_inputs():
    """Seed 0: probabilities softmax(N(0,2) + 0.002 * position) per (layer,
    28 q-heads, token); K/V N(0,1) fp16; a 16-step history in which every
    slab has min(Poisson(3), 16) hits with uniform weights."""
    w = C1
    nb = w["T"] // w["tpb"]
    n = w["L"] * w["Hkv"] * nb
    rng = np.random.default_rng(0)
    logits = (rng.normal(0, 2, (w["L"], w["Hq"], w["T"])).astype(np.float32)
              + (0.002 * np.arange(w["T"])).astype(np.float32))
    logits -= logits.max(-1, keepdims=True)
    p = np.exp(logits)
    probs = (p / p.sum(-1, keepdims=True)).astype(np.float32)
    kv = rng.standard_normal((w["L"], 2, w["Hkv"], w["T"], w["D"])).astype(np.float16)
    hits = np.minimum(rng.poisson(3, n), w["hist"])
    history = [([], []) for _ in range(w["hist"])]
    for i in range(n):
        for s, x in zip(rng.choice(w["hist"], hits[i], replace=False),
                        rng.random(hits[i]).astype(np.float32)):
            history[int(s)][0].append(i)
            history[int(s)][1].append(float(x))
    return probs, kv, history


def run_cpu_step(args, torch, okv):
    """One request, 8 layers x 4 KV heads, 64-token blocks, 4096 tokens (2,048
    slabs of 32 KB), after a 16-step hit history.  A step: report the
    probabilities (one launch), step + classify, select the coldest 50%, evict
    them to pinned DRAM and promote them back, read the counts -- device time
    per step (events) and wall time per step with the host waiting for the
    counts.  Beside it (unless --no-cpu-baseline) the reference's own path for
    the same step on one host core: the C restatement of the managers'
    reduction, the reference scheduler (attn_tracker_update_batch,
    tm_step_done, tm_schedule_once, coldest-first order) and its data plane
    evicting and promoting block by block."""
    w = C1
    nb = w["T"] // w["tpb"]
    n = w["L"] * w["Hkv"] * nb
    slab = w["tpb"] * w["D"] * 2 * 2
    k = int(w["evict_frac"] * n)
    probs, kv, history = _c1_inputs()
    L = okv.lib()
    cfg = okv.make_config(gpu_pool_bytes=(n + 64) * slab, dram_pool_bytes=n * slab,
                          tokens_per_block=w["tpb"], d_head=w["D"], dtype=0,
                          device=torch.cuda.current_device(), max_blocks_per_head=nb + 8)
    ext = okv.OrchkvConfigExt()
    ext.max_blocks = 4096
    assert L.orchkv_init_ext(C.byref(cfg), C.byref(ext)) == 0
    stream = torch.cuda.current_stream()
    L.orchkv_set_stream(C.c_void_p(stream.cuda_stream))
    tm = okv.Manager(tracker_cap=4096, max_blocks=8192, ema_lambda=0.9, alpha=0.5, beta=0.3,
                     gamma=0.2, recency_tau=50.0, cooldown_sec=0.0)
    assert L.orchkv_attach_scheduler(tm.ref) == 0
    ctx = L.orchkv_request_create(0, w["L"], w["Hkv"])
    for layer in range(w["L"]):
        assert L.orchkv_prefill(ctx, layer, kv[layer, 0].ctypes.data, kv[layer, 1].ctypes.data,
                                w["T"]) == 0
    arr = (C.c_void_p * 1)(ctx)
    ids = torch.empty(n, dtype=torch.int32, device="cuda")
    assert L.orchkv_block_id_table(arr, 1, w["T"], C.c_void_p(ids.data_ptr())) == 0
    for sl, wt in history:
        if sl:
            hid = ids[torch.as_tensor(sl, device="cuda")].contiguous()
            hw = torch.as_tensor(wt, dtype=torch.float32, device="cuda")
            assert L.tm_report_attn_batch_dev(tm.ref, C.c_void_p(hid.data_ptr()),
                                              C.c_void_p(hw.data_ptr()), len(sl)) == 0
        assert L.tm_step_and_classify(tm.ref) == 0
    dprobs = torch.from_numpy(probs).cuda()
    victims = torch.empty(n, dtype=torch.int32, device="cuda")
    counts = torch.zeros(8, dtype=torch.int32, device="cuda")
    h_counts = torch.zeros(8, dtype=torch.int32).pin_memory()
    vp = lambda t, off=0: C.c_void_p(t.data_ptr() + off)   # noqa: E731

    def step():
        assert L.tm_report_attn_probs(tm.ref, vp(dprobs), w["L"], w["Hq"], w["Hkv"], w["T"],
                                      w["tpb"], None, vp(ids)) == 0
        assert L.tm_step_and_classify(tm.ref) == 0
        assert L.tm_select_victims(tm.ref, k, vp(victims), vp(counts)) == 0
        assert L.orchkv_evict_batch_to_dram(vp(victims), vp(counts), n, vp(counts, 8)) == 0
        assert L.orchkv_promote_batch_to_gpu(vp(victims), vp(counts), n, vp(counts, 16)) == 0
        h_counts.copy_(counts, non_blocking=True)
        stream.synchronize()

    for _ in range(max(args.warmup, 3)):
        step()
    dev_us, wall_us = [], []
    for _ in range(max(args.steps, 10)):
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0 = time.perf_counter()
        e0.record()
        step()
        e1.record()
        e1.synchronize()
        wall_us.append((time.perf_counter() - t0) * 1e6)
        dev_us.append(e0.elapsed_time(e1) * 1e3)
    c = h_counts.tolist()
    assert c[0] == k and c[2] == k and c[4] == k, c
    L.orchkv_request_destroy(ctx)
    tm.close()
    L.orchkv_shutdown()
    out = {"workload": w["name"], "blocks": n, "evicted_and_promoted": k,
           "us_per_step_device": round(statistics.median(dev_us), 1),
           "us_per_step_wall": round(statistics.median(wall_us), 1),
           "steps": len(dev_us),
           "note": "median over steps; wall time includes the host waiting for the counts"}
    if not args.no_cpu_baseline:
        out["cpu_baseline"] = _c1_reference(probs, kv, history, k)
    return out


def _c1_reference(probs, kv, history, k):
    """The reference's own path for the step above, on one host core
    (oracle/_ref: its scheduler and data plane compiled from its sources)."""
    from oracle import oracle as O
    if not O.ref_available():
        return None
    w = C1
    nb = w["T"] // w["tpb"]
    n = w["L"] * w["Hkv"] * nb
    slab = w["tpb"] * w["D"] * 2 * 2
    R = O.ref()
    rtm = O.RefTM(tracker_cap=4096, max_blocks=8192, ema_lambda=0.9, alpha=0.5, beta=0.3,
                  gamma=0.2, recency_tau=50.0, cooldown_sec=0.0)
    rtm.register_range(n)
    ids = np.arange(n, dtype=np.uint64)
    for sl, wt in history:
        if sl:
            rtm.report_batch(ids[sl], np.asarray(wt, np.float32))
        rtm.step_done()
    assert R.ref_api_init(0, (n + 64) * slab, n * slab, w["tpb"], w["D"], 0, 4, nb + 8,
                          b"/dev/shm/orchkv_ref_c1") == 0
    ctx = R.ref_api_request_create(0, w["L"], w["Hkv"])
    for layer in range(w["L"]):
        assert R.ref_api_prefill(ctx, layer, kv[layer, 0].ctypes.data, kv[layer, 1].ctypes.data,
                                 w["T"]) == 0
    vict = np.zeros(k, np.uint64)
    times = []
    for s in range(6):
        t0 = time.perf_counter()
        mass = O.score_blocks(probs, w["Hq"], w["Hkv"], w["tpb"]).reshape(-1)
        c = R.ref_arm_sched_step(rtm.h, ids, mass.copy(), n, 1.0, k, vict, np.zeros(3))
        v = vict[:c].astype(np.int64)
        lhb = np.stack([v // (w["Hkv"] * nb), (v // nb) % w["Hkv"], v % nb], 1).astype(np.uint32)
        tmp = np.zeros(2)
        assert R.ref_api_migrate_list(ctx, lhb.reshape(-1), c, 0, tmp) == 0
        assert R.ref_api_migrate_list(ctx, lhb.reshape(-1), 0, c, tmp) == 0
        if s:
            times.append((time.perf_counter() - t0) * 1e6)
    R.ref_api_request_destroy(ctx)
    R.ref_api_shutdown()
    rtm.close()
    return {"kind": "reference", "cores": 1, "us_per_step": round(statistics.median(times), 1),
            "sample": "the whole configuration (one request), median of 5 steps after one"}


def score_bytes(wl):
    """Algorithmic bytes of one scoring launch: probabilities read once, block
    id table read, per-block tracker read (active, sum, max) and written (sum,
    max, last hit)."""
    probs = wl.rows * wl.Hq * wl.T * 4
    per_block = 4 + 1 + 4 + 4 + 4 + 4 + 8
    return probs + wl.n_blocks * per_block


def pack_roofline(launch_ms, total_bytes, hbm_peak, peak_kind):
    """The kernel with the largest share of device time in a step: the evict
    pack (HBM gather of the victims into the staging ring).  achieved =
    algorithmic bytes (each packed slab read once and written once) per
    launch / the mean launch time from CUDA events around each launch of the
    timed steps; it runs while the copy engine drains earlier chunks to the
    host."""
    if not launch_ms:
        return None
    n = len(launch_ms)
    per_launch = total_bytes / n
    ms = sum(launch_ms) / n
    achieved = per_launch / (ms * 1e-3) / 1e9
    return {"kernel": "evict pack (HBM gather -> staging ring), the largest share of "
                      "device time per step", "bound": "hbm",
            "achieved": round(achieved, 1), "peak": hbm_peak, "unit": "GB/s",
            "frac": round(achieved / hbm_peak, 4), "peak_kind": peak_kind,
            "nominal_peak": NOMINAL_HBM_GBS, "frac_nominal": round(achieved / NOMINAL_HBM_GBS, 4),
            "bytes_per_launch": round(per_launch), "ms_per_launch": round(ms, 4),
            "launches": n,
            "traffic": round(PACK_TRAFFIC_PER_FULL_LAUNCH * per_launch / PACK_FULL_LAUNCH_BYTES),
            "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum of one "
                              "full-chunk launch, scaled by bytes per launch"}


def unpack_launches(L):
    """Per-launch device times (ms) of the last promote's unpack kernels and
    the bytes they moved in total."""
    ms, nb, n = (C.c_float * 64)(), (C.c_ulonglong * 64)(), C.c_uint32()
    L.orchkv_last_unpack_chunks(ms, nb, 64, C.byref(n))
    k = min(64, n.value)
    return [ms[i] for i in range(k)], sum(nb[i] for i in range(k))


def pack_launches(L):
    """Per-launch device times (ms) of the last staged evict's pack kernels
    and the bytes they read and wrote in total."""
    ms, nbytes, chunks, pr = C.c_float(), C.c_ulonglong(), C.c_uint32(), C.c_float()
    L.orchkv_last_migration_profile(C.byref(ms), C.byref(nbytes), C.byref(chunks), C.byref(pr))
    arr, n = (C.c_float * 64)(), C.c_uint32()
    L.orchkv_last_pack_chunks(arr, 64, C.byref(n))
    return [arr[i] for i in range(min(64, n.value))], nbytes.value


def pack_first_chunk(chunk_ms, total_bytes, chunks, hbm_peak):
    """The first staging chunk's pack, timed before the copy engine starts
    draining the evict (full chunks carry equal bytes): ms, GB/s and the
    fraction of the measured HBM peak."""
    if not chunk_ms or chunks < 2:
        return None
    nbytes = total_bytes / chunks
    gbs = nbytes / max(chunk_ms[0], 1e-9) / 1e6
    return {"ms": round(chunk_ms[0], 4), "achieved_gbs": round(gbs, 1),
            "frac": round(gbs / hbm_peak, 4),
            "later_chunks_ms_mean": round(sum(chunk_ms[1:]) / (len(chunk_ms) - 1), 4)}


def hook_blockmean_probe(torch, okv, hbm_peak, passes=3, warm=2):
    """The vLLM hook's block-mean reduction (tm_report_attn_blockmean) on the
    workload's decode-step attention weights: bf16 [requests, q_heads, 1,
    context] per layer, one call per layer over distinct buffers (28 x 14.7
    MB, larger than L2), timed with events on torch's current stream (the
    probe's own manager is bound to it).  Timed twice: scores only (the
    reduction kernel alone), and with every (head, block) reported to a
    registered tracker id, as the hook's default mode does (reduction +
    tracker apply)."""
    B, Hq, T, tpb, Ly = WL["B"], WL["Hq"], WL["T"], WL["tpb"], WL["L"]
    nb = (T + tpb - 1) // tpb
    L = okv.lib()
    m = okv.Manager(tracker_cap=1 << 15, max_blocks=1 << 15)
    assert L.tm_set_stream(m.ref, C.c_void_p(torch.cuda.current_stream().cuda_stream)) == 0
    for i in range(Hq * nb):
        assert m.register_id(i) == 0
    ids = torch.arange(Hq * nb, dtype=torch.int32, device="cuda")
    g = torch.Generator(device="cuda").manual_seed(77)
    ws = [torch.softmax(torch.randn(B, Hq, 1, T, generator=g, device="cuda") * 2.0,
                        dim=-1).to(torch.bfloat16) for _ in range(Ly)]
    sc = torch.empty(Ly, Hq, nb, device="cuda")

    def timed(id_ptr):
        def one_pass():
            for i, w in enumerate(ws):
                assert L.tm_report_attn_blockmean(m.ref, C.c_void_p(w.data_ptr()), 1, B, Hq, 1, T,
                                                  tpb, id_ptr,
                                                  C.c_void_p(sc[i].data_ptr())) == 0
        for _ in range(warm):
            one_pass()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(passes):
            one_pass()
        e1.record()
        e1.synchronize()
        return e0.elapsed_time(e1) / (passes * Ly)

    ms = timed(None)
    ms_rep = timed(C.c_void_p(ids.data_ptr()))
    m.close()
    n = passes * Ly
    nbytes = B * Hq * T * 2 + Hq * nb * 4
    del ws, sc, ids
    return {"kernel": "hook block mean (tm_report_attn_blockmean, scores only)",
            "shape": f"bf16 [{B}, {Hq}, 1, {T}] per layer, block {tpb}, {Ly} layers",
            "launches": n, "ms_per_launch": round(ms, 4), "bytes_per_launch": nbytes,
            "achieved_gbs": round(nbytes / ms / 1e6, 1),
            "frac": round(nbytes / ms / 1e6 / hbm_peak, 4),
            "ms_per_layer_with_reports": round(ms_rep, 4)}


def run_ours(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist

    torch.cuda.set_device(local_rank)
    import orchkv_b200 as okv
    okv.lib()
    comm = None
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120),
                                device_id=torch.device("cuda", local_rank))
        uid = (C.c_ubyte * 128)()
        if rank == 0:
            assert okv.lib().orchkv_comm_unique_id(uid) == 0
        buf = torch.tensor(list(bytes(uid)), dtype=torch.uint8, device="cuda")
        dist.broadcast(buf, 0)
        uid = (C.c_ubyte * 128)(*buf.cpu().tolist())
        comm = okv.lib().orchkv_comm_create(rank, world, uid, 60.0)
        assert comm, "NCCL communicator creation failed"

    # one dedicated stream for torch ops and the library (non-default, so
    # events and copies order with every kernel the library launches)
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    wl = Workload(torch, okv, rank, world, comm)
    hbm_peak, peak_kind = peaks()

    def barrier():
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    link = host_link_probe(torch, barrier=barrier if world > 1 else None)
    for _ in range(args.warmup):
        wl.step()
        wl.restore()
    # timed: K steps, each bracketed by barrier + synchronize; the restore of
    # the DRAM-resident remainder runs outside the brackets
    step_ms, phase_acc, score_ms, report_pass_ms = [], {}, [], []
    pack_ms_acc, pack_bytes_acc = [], 0
    unpack_ms_acc, unpack_bytes_acc = [], 0
    migrated = 0
    launches0 = okv.lib().orchkv_kernel_launches()
    xch_ms, xch_calls = C.c_float(), C.c_uint32()
    if comm:                                  # drop the warm-up's exchanges
        okv.lib().orchkv_comm_exchange_time(comm, C.byref(xch_ms), C.byref(xch_calls))
    xch = [0.0, 0]
    with ClockSampler(local_rank) as clk:
        launches_timed = 0
        la = launches0
        for _ in range(args.steps):
            barrier()
            la = okv.lib().orchkv_kernel_launches()
            t0 = torch.cuda.Event(enable_timing=True)
            t1 = torch.cuda.Event(enable_timing=True)
            t0.record()
            wl.step()
            t1.record()
            barrier()
            step_ms.append(t0.elapsed_time(t1))
            ph = wl.phases()
            for k, v in ph.items():
                phase_acc.setdefault(k, []).append(v)
            mk, sc, od = C.c_float(), C.c_float(), C.c_float()
            assert wl.L.tm_last_report_times(wl.tm.ref, C.byref(mk), C.byref(sc), C.byref(od)) == 0
            score_ms.append(sc.value)
            report_pass_ms.append((mk.value, od.value))
            c = wl.h_counts.tolist()
            migrated += c[2] + c[4]
            launches_timed += okv.lib().orchkv_kernel_launches() - la
            # this step's pack and unpack launches, timed by events around each
            pk = pack_launches(wl.L)
            pack_ms_acc.extend(pk[0])
            pack_bytes_acc += pk[1]
            up = unpack_launches(wl.L)
            unpack_ms_acc.extend(up[0])
            unpack_bytes_acc += up[1]
            if comm:
                okv.lib().orchkv_comm_exchange_time(comm, C.byref(xch_ms), C.byref(xch_calls))
                xch[0] += xch_ms.value
                xch[1] += xch_calls.value
            wl.restore()
            la = okv.lib().orchkv_kernel_launches()
    # e2e through the C ABI with host inputs (one untimed step first: the
    # library sizes its staging for host inputs on first use)
    wl.step(e2e=True)
    wl.restore()
    e2e_ms, e2e_ph = [], {}
    for _ in range(max(1, min(args.steps, 5))):
        barrier()
        t0 = torch.cuda.Event(enable_timing=True)
        t1 = torch.cuda.Event(enable_timing=True)
        t0.record()
        wl.step(e2e=True)
        t1.record()
        barrier()
        e2e_ms.append(t0.elapsed_time(t1))
        for k, v in wl.phases().items():
            e2e_ph.setdefault(k, []).append(v)
        c_e2e = wl.h_counts.tolist()
        wl.restore()
    assert wl.L.tm_stage_input_async(wl.tm.ref, None, 0) == 0      # the last step's upload
    # pack kernel profile of one more evict (device events on its stream)
    wl.step()
    pk_ms, pk_bytes, pk_chunks, pr_ms = C.c_float(), C.c_ulonglong(), C.c_uint32(), C.c_float()
    wl.L.orchkv_last_migration_profile(C.byref(pk_ms), C.byref(pk_bytes), C.byref(pk_chunks),
                                       C.byref(pr_ms))
    # per-chunk pack times: chunk 0 is packed before any device-to-host copy
    # of the evict is in flight, the later ones while the copy engine drains
    chunk_ms = (C.c_float * 64)()
    n_chunk_ms = C.c_uint32()
    wl.L.orchkv_last_pack_chunks(chunk_ms, 64, C.byref(n_chunk_ms))
    chunk_ms = [chunk_ms[i] for i in range(min(64, n_chunk_ms.value))]
    lay = [C.c_uint32() for _ in range(3)]
    wl.L.orchkv_last_evict_layout(*[C.byref(x) for x in lay])
    play = [C.c_uint32() for _ in range(3)] + [C.c_int()]
    wl.L.orchkv_last_promote_layout(*[C.byref(x) for x in play])
    c_last = wl.h_counts.tolist()
    wl.restore()
    hook = hook_blockmean_probe(torch, okv, hbm_peak)

    mean_ms = sum(step_ms) / len(step_ms)
    per_step_migrated = migrated / args.steps
    if world > 1:
        t = torch.tensor([mean_ms, per_step_migrated, sum(e2e_ms) / len(e2e_ms)],
                         dtype=torch.float64, device="cuda")
        mx = t.clone()
        dist.all_reduce(mx, op=dist.ReduceOp.MAX)
        sm = t.clone()
        dist.all_reduce(sm, op=dist.ReduceOp.SUM)
        mean_ms_max, migrated_total, e2e_max = float(mx[0]), float(sm[1]), float(mx[2])
    else:
        mean_ms_max, migrated_total, e2e_max = mean_ms, per_step_migrated, sum(e2e_ms) / len(e2e_ms)

    sb = score_bytes(wl)
    score_avg = sum(score_ms) / len(score_ms)
    achieved = sb / (score_avg * 1e-3) / 1e9
    phases = {k: round(sum(v) / len(v), 4) for k, v in phase_acc.items()}
    evict_bytes = c_last[2] * wl.slab
    promote_bytes = c_last[4] * wl.slab
    # each rank's host-link bound of its swap (its synchronized probe), and
    # the box's: every rank moves its own bytes at its share at once
    bound_ms = 1e3 * max(evict_bytes / (link["d2h"] * 1e9), promote_bytes / (link["h2d"] * 1e9),
                         (evict_bytes + promote_bytes) / (link["both"] * 1e9))
    lt = torch.tensor([link["d2h"], link["h2d"], bound_ms], dtype=torch.float64, device="cuda")
    if world > 1:
        lall = [torch.zeros_like(lt) for _ in range(world)]
        dist.all_gather(lall, lt)
        lall = [x.tolist() for x in lall]
    else:
        lall = [lt.tolist()]
    line = None
    if rank == 0:
        cpu = None
        if world == 1 and not args.no_cpu_baseline:
            cpu = cpu_baseline_sample(args)
        line = {
            "metric": METRIC,
            "value": round(migrated_total / (mean_ms_max * 1e-3), 1),
            "unit": "blocks/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(mean_ms_max, 4),
            "us_per_step": round(mean_ms_max * 1e3, 1),
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "f32+bf16",          # scores, EMA and hotness in f32; KV slabs moved as bf16
            "data": "synthetic (seeded: logits N(0,2) + 1% heavy hitters, KV N(0,1))",
            "config": {"workload": WL["name"], "requests": WL["B"], "context": WL["T"],
                       "layers": WL["L"], "q_heads": WL["Hq"], "kv_heads": WL["Hkv"],
                       "d_head": WL["D"], "tokens_per_block": WL["tpb"],
                       "blocks_per_gpu": wl.n_blocks, "evict_frac": EVICT_FRAC,
                       "promote_frac": PROMOTE_FRAC, "parallelism": (f"replica x{world}: every rank holds the whole "
                                       f"workload, selections global over ranks"
                                       if world > 1 else "single GPU"),
                       "value_scope": "all ranks' migrated blocks per second (whole job)",
                       "l2": "inputs larger than L2 (0.82 GB probs, 14 GiB KV pool)"},
            "gpu_launches": int(launches_timed),
            "gpu_launches_per_step": round(launches_timed / args.steps, 1),
            "roofline": pack_roofline(pack_ms_acc, pack_bytes_acc, hbm_peak, peak_kind),
            "unpack": ({"kernel": "promote unpack (H2D staging ring -> GPU slabs)",
                        "launches": len(unpack_ms_acc),
                        "ms_per_launch": round(sum(unpack_ms_acc) / len(unpack_ms_acc), 4),
                        "bytes_per_launch": round(unpack_bytes_acc / len(unpack_ms_acc)),
                        "achieved_gbs": round(unpack_bytes_acc / sum(unpack_ms_acc) / 1e6, 1),
                        "frac": round(unpack_bytes_acc / sum(unpack_ms_acc) / 1e6 / hbm_peak, 4)}
                       if unpack_ms_acc else None),
            "roofline_score": {
                "kernel": "score (per-block attention mass, tm_report_attn_probs)",
                "bound": "hbm", "achieved": round(achieved, 1), "peak": hbm_peak,
                "unit": "GB/s", "frac": round(achieved / hbm_peak, 4),
                "peak_kind": peak_kind, "nominal_peak": NOMINAL_HBM_GBS,
                "frac_nominal": round(achieved / NOMINAL_HBM_GBS, 4), "bytes_per_launch": sb,
                "ms_per_launch": round(score_avg, 4),
                "traffic": round(SCORE_TRAFFIC_PER_REQUEST * WL["B"]),
                "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum of one "
                                  "8-request launch, scaled by requests"},
            "report_passes": {
                "duplicate_slot_pass_ms": round(sum(x[0] for x in report_pass_ms)
                                                / len(report_pass_ms), 4),
                "ordered_pass_ms": round(sum(x[1] for x in report_pass_ms)
                                         / len(report_pass_ms), 4),
                "note": "tm_report_attn_probs = duplicate-slot pass + score kernel + ordered "
                        "pass (returns at once when no slot repeats); the score phase covers "
                        "all three"},
            "hook": hook,
            "pack": {"kernel": "evict pack (HBM gather -> staging)",
                     "ms": round(pk_ms.value, 4), "bytes": pk_bytes.value,
                     "achieved_gbs": round(pk_bytes.value / max(pk_ms.value, 1e-9) / 1e6, 1),
                     "frac": round(pk_bytes.value / max(pk_ms.value, 1e-9) / 1e6 / hbm_peak, 4),
                     "first_chunk": pack_first_chunk(chunk_ms, pk_bytes.value, pk_chunks.value,
                                                     hbm_peak),
                     "chunks": pk_chunks.value, "dram_runs": lay[0].value,
                     "ce_copies": lay[1].value, "zero_copy_blocks": lay[2].value},
            "host_link": {
                "swap_ms": phases.get("swap"), "overlapped": bool(play[3].value),
                "evict_bytes": evict_bytes,
                "evict_gbs": round(evict_bytes / max(phases.get("swap", 1), 1e-9) / 1e6, 1),
                "promote_bytes": promote_bytes, "promote_ms": round(pr_ms.value, 3),
                "promote_gbs": round(promote_bytes / max(pr_ms.value, 1e-9) / 1e6, 1),
                "promote_dram_runs": play[0].value, "promote_ce_copies": play[1].value,
                "promote_zero_copy_blocks": play[2].value,
                "both_gbs": round((evict_bytes + promote_bytes)
                                  / max(phases.get("swap", 1), 1e-9) / 1e6, 1),
                "measured_ce_d2h_gbs": link["d2h"], "measured_ce_h2d_gbs": link["h2d"],
                "measured_ce_both_gbs": link["both"],
                # host-link bound of the swap: each direction at its measured
                # rate, both together at most at the measured two-way rate
                "bound_ms": round(1e3 * max(evict_bytes / (link["d2h"] * 1e9),
                                            promote_bytes / (link["h2d"] * 1e9),
                                            (evict_bytes + promote_bytes) / (link["both"] * 1e9)), 3),
                "frac": round(1e3 * max(evict_bytes / (link["d2h"] * 1e9),
                                        promote_bytes / (link["h2d"] * 1e9),
                                        (evict_bytes + promote_bytes) / (link["both"] * 1e9))
                              / max(phases.get("swap", 1), 1e-9), 4)},
            "box_host_link": {
                "probe_d2h_gbs_per_rank": [round(x[0], 1) for x in lall],
                "probe_d2h_gbs_summed": round(sum(x[0] for x in lall), 1),
                "probe_h2d_gbs_summed": round(sum(x[1] for x in lall), 1),
                "bound_ms_max_rank": round(max(x[2] for x in lall), 3),
                "ceiling_blocks_s": round(migrated_total / (max(x[2] for x in lall) * 1e-3), 1),
                "note": "every rank probes at once; the ceiling is the whole job's migrated "
                        "blocks over the slowest rank's host-link bound"},
            "phases_ms": phases,
            "collective": ({"kind": "ncclAllReduce of 16 KB key histograms + ncclAllGather "
                                    "of tie counts inside each global selection",
                            "exchanges_per_step": round(xch[1] / args.steps, 1),
                            "device_ms_per_step": round(xch[0] / args.steps, 4)}
                           if comm else None),
            "e2e": {"value": round(migrated_total / (e2e_max * 1e-3), 1), "unit": "blocks/s",
                    "ms_per_step": round(e2e_max, 4),
                    "input_pipelining": "each step uploads the next step's host probabilities "
                                        "(tm_stage_input_async) while its swap runs; the "
                                        "next step's report reads that copy",
                    "phases_ms_rank0": {k: round(sum(v) / len(v), 4) for k, v in e2e_ph.items()},
                    "h2d_bytes_per_step": int(wl.probs.numel() * 4 + wl.tok.numel() * 2
                                              + c_e2e[4] * wl.slab),
                    "d2h_bytes_per_step": int(c_e2e[2] * wl.slab + 32)},
            "clocks": clk.summary(),
        }
        if cpu:
            line["cpu_baseline"] = cpu
    wl.close()
    del wl
    torch.cuda.empty_cache()
    if not args.no_sharded:
        sharded = run_sharded(args, torch, okv, rank, world, comm, dist if world > 1 else None,
                              link["d2h"])
        if line is not None:
            line["sharded"] = sharded
        torch.cuda.empty_cache()
    if not args.no_multiplexed:
        mx = run_multiplexed(args, torch, okv, rank, world, dist if world > 1 else None, link)
        if line is not None:
            line["multiplexed"] = mx
    if not args.no_three_tier:
        tt = run_three_tier(args, torch, okv, rank, world, comm, dist if world > 1 else None)
        if line is not None:
            line["three_tier"] = tt
        torch.cuda.empty_cache()
    if world == 1 and not args.no_cpu_step:
        line["cpu_step"] = run_cpu_step(args, torch, okv)
    if comm:
        okv.lib().orchkv_comm_destroy(comm)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if line:
        print(json.dumps(line), flush=True)


def host_link_probe(torch, nbytes=512 << 20, reps=3, barrier=None):
    """Copy-engine bandwidth of this GPU's host link with pinned memory, in
    GB/s: each direction alone, and both at once on two streams (bytes moved
    in both directions over the time of the pair).  Best of `reps`.  With
    several ranks, `barrier` starts every rep on all ranks together, so each
    rep measures this rank's share while every rank copies."""
    h = torch.empty(nbytes, dtype=torch.uint8).pin_memory()
    d = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
    h2 = torch.empty(nbytes, dtype=torch.uint8).pin_memory()
    d2 = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
    s1, s2 = torch.cuda.Stream(), torch.cuda.Stream()
    out = {}
    for name, pairs in (("h2d", [(d, h)]), ("d2h", [(h, d)]), ("both", [(d, h), (h2, d2)])):
        best = 0.0
        for _ in range(reps):
            if barrier:
                barrier()
            torch.cuda.synchronize()
            a = torch.cuda.Event(enable_timing=True)
            b = torch.cuda.Event(enable_timing=True)
            a.record()
            for (dst, src), st in zip(pairs, (s1, s2)):
                st.wait_event(a)
                with torch.cuda.stream(st):
                    dst.copy_(src, non_blocking=True)
            for st in (s1, s2)[:len(pairs)]:
                torch.cuda.current_stream().wait_stream(st)
            b.record()
            b.synchronize()
            best = max(best, len(pairs) * nbytes / (a.elapsed_time(b) * 1e-3) / 1e9)
        out[name] = round(best, 1)
    del h, d, h2, d2
    return out


# ---------------------------------------------------------------------------
# Reference arm: the reference's C scheduler + per-block migration on a sample
# ---------------------------------------------------------------------------

def host_threads():
    """Host cores this process may run on."""
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def _reference_sample(steps=3, warm=1, threads=1):
    """Time the reference on `threads` request(s) of the workload, one request
    per host thread, in the same steady state: 5% of the blocks (the coldest
    at the start) held in DRAM.  A step: fixed-order C reduction of the
    attention probabilities (restating the managers' torch reduction; one
    request per thread), attn_tracker_update_batch + tm_step_done +
    tm_schedule_once (reference C; one manager, so one thread), the
    FastKVCacheManager coldest-first order over the blocks on the GPU, then
    orchkv_evict_to_dram per victim (25% of the blocks), orchkv_promote_to_gpu
    per reserve block and orchkv_append_token per (request, layer), through
    the reference's own orchkv_api (real CUDA copies).  The reference's data
    plane takes a lock around each shared pool and its transfer engine, and
    its per-request state belongs to one request, so the threads migrate
    their own requests concurrently (src/tiered_store/gpu_tier.cu:65-93,
    src/tiered_store/transfer.cu:62-92); the transfer engine gets one CUDA
    stream per thread (its num_cuda_streams setting).  Each phase is timed by
    the wall clock.  Returns blocks/s (migrated) and details."""
    from concurrent.futures import ThreadPoolExecutor

    import numpy as np

    from oracle import oracle as O
    w = WL
    B, Ly, Hq, Hkv, D, T, tpb = threads, w["L"], w["Hq"], w["Hkv"], w["D"], w["T"], w["tpb"]
    nb = T // tpb
    n = B * Ly * Hkv * nb
    slab = tpb * D * 4
    rng = np.random.default_rng(0)
    logits = rng.normal(0, 2, (B * Ly, Hq, T)).astype(np.float32)
    for r in range(B * Ly):
        for h in range(Hq):
            logits[r, h, rng.choice(T, T // 100, replace=False)] += 6.0
    logits -= logits.max(-1, keepdims=True)
    np.exp(logits, out=logits)
    logits /= logits.sum(-1, keepdims=True)
    probs = logits
    del logits
    R = O.ref()
    tm = O.RefTM(tracker_cap=n, max_blocks=n, ema_lambda=0.9, alpha=0.5, beta=0.3, gamma=0.2,
                 recency_tau=50.0, cooldown_sec=0.0)
    ids = np.arange(n, dtype=np.uint64)
    tm.register_range(n)
    # tm_schedule_once's prefetch scan takes n_blocks x 16 bytes with alloca
    # (src/scheduler/tiered_manager.c:283-291): past ~500k blocks that is more
    # than a default 8 MiB stack, so the scheduler runs on one thread whose
    # stack holds it.
    old_stack = threading.stack_size(max(64 << 20, 2 * 16 * n + (32 << 20)))
    sched_pool = ThreadPoolExecutor(1)
    sched_pool.submit(lambda: None).result()
    threading.stack_size(old_stack)

    def sched(wts, k, out):
        return sched_pool.submit(R.ref_arm_sched_step, tm.h, ids, wts, n, 0.95, k, out,
                                 np.zeros(3)).result()
    gpu_pool = (n + B * Ly * Hkv * 8 + 64) * slab
    dram_pool = (n // 4 + n // 20 + 128) * slab
    rc = R.ref_api_init(0, gpu_pool, dram_pool, tpb, D, 1, max(4, threads), nb + 8,
                        b"/dev/shm/orchkv_ref_bench")
    assert rc == 0, rc
    kv = rng.standard_normal((Hkv, T, D)).astype(np.float16)
    ctxs = []
    for b in range(B):
        c = R.ref_api_request_create(b, Ly, Hkv)
        for layer in range(Ly):
            assert R.ref_api_prefill(c, layer, kv.ctypes.data, kv.ctypes.data, T) == 0
        ctxs.append(c)
    tok = np.zeros((Hkv, D), np.float16)
    k_e, k_p = int(EVICT_FRAC * n), int(PROMOTE_FRAC * n)
    pool = ThreadPoolExecutor(threads) if threads > 1 else None

    def pmap(fn, items):
        items = list(items)
        return list(pool.map(fn, items)) if pool else [fn(x) for x in items]

    def by_request(id_list):
        """block ids -> {request: uint32 [(layer, head, block), ...]} in list order"""
        v = np.asarray(id_list, np.int64)
        b, rem = np.divmod(v, Ly * Hkv * nb)
        layer, rem = np.divmod(rem, Hkv * nb)
        head, bi = np.divmod(rem, nb)
        lhb = np.stack([layer, head, bi], axis=1).astype(np.uint32)
        order = np.argsort(b, kind="stable")
        bs, starts = np.unique(b[order], return_index=True)
        ends = list(starts[1:]) + [len(order)]
        return {int(r): np.ascontiguousarray(lhb[order[s:e]]) for r, s, e in zip(bs, starts, ends)}

    def migrate(groups, evict):
        def one(item):
            b, arr = item
            tmp = np.zeros(2)
            k = len(arr)
            rc = R.ref_api_migrate_list(ctxs[b], arr.reshape(-1), k if evict else 0,
                                        0 if evict else k, tmp)
            assert rc == 0, rc
        t0 = time.perf_counter()
        pmap(one, groups.items())
        return time.perf_counter() - t0

    def score():
        return np.concatenate(pmap(
            lambda b: O.score_blocks(probs[b * Ly:(b + 1) * Ly], Hq, Hkv, tpb), range(B)))

    def append(b):
        for layer in range(Ly):
            assert R.ref_api_append(ctxs[b], layer, tok.ctypes.data, tok.ctypes.data) == 0

    # the DRAM-resident reserve: one scheduler pass, the coldest 5% evicted
    # and marked as off the GPU (the manager's tm_set_block_tier bookkeeping)
    reserve = np.zeros(k_p, np.uint64)
    w0 = score()
    c_p = sched(w0.reshape(-1).copy(), k_p, reserve)
    reserve = reserve[:c_p].copy()
    tm.set_tiers(reserve, 1)
    res_groups = by_request(reserve)
    migrate(res_groups, evict=True)
    vict = np.zeros(k_e, np.uint64)
    times = []
    for s in range(warm + steps):
        t0 = time.perf_counter()
        w_ = score()                                          # [B*Ly, Hkv, nb]
        t1 = time.perf_counter()
        c = sched(w_.reshape(-1).copy(), k_e, vict)
        t2 = time.perf_counter()
        groups = by_request(vict[:c])
        t3 = time.perf_counter()
        evict_s = migrate(groups, evict=True)
        promote_s = migrate(res_groups, evict=False)
        t4 = time.perf_counter()
        pmap(append, range(B))
        t5 = time.perf_counter()
        # back to the starting state (not timed)
        migrate(groups, evict=False)
        migrate(res_groups, evict=True)
        step_s = (t1 - t0) + (t2 - t1) + (t3 - t2) + evict_s + promote_s + (t5 - t4)
        if s >= warm:
            times.append(dict(step_s=step_s, score_s=t1 - t0, sched_s=t2 - t1,
                              group_s=t3 - t2, evict_s=evict_s, promote_s=promote_s,
                              append_s=t5 - t4, migrated=c + len(reserve), blocks=n))
    if pool:
        pool.shutdown()
    sched_pool.shutdown()
    for cx in ctxs:
        R.ref_api_request_destroy(cx)
    R.ref_api_shutdown()
    tm.close()
    mean = {k: sum(t[k] for t in times) / len(times) for k in times[0]}
    return mean


def cpu_baseline_sample(args):
    from oracle import oracle as O
    if not O.ref_available():
        return None
    m = _reference_sample(steps=max(1, min(args.steps, 3)))
    return {"value": round(m["migrated"] / m["step_s"], 1), "unit": "blocks/s",
            "cores": 1, "kind": "reference",
            "sample": f"1 of {WL['B']} requests ({int(m['blocks'])} blocks): reference C scheduler "
                      f"(attn_tracker_update_batch, tm_step_done, tm_schedule_once) + "
                      f"coldest-25% order + per-block orchkv_evict_to_dram of the victims / "
                      f"orchkv_promote_to_gpu of the 5% DRAM reserve + orchkv_append_token, "
                      f"mean of {max(1, min(args.steps, 3))} steps",
            "us_per_step_sample": round(m["step_s"] * 1e6, 1),
            "phases_s": {k: round(v, 6) for k, v in m.items() if k.endswith("_s")},
            "cpu_pack_gbs": cpu_pack_gbs()}


def cpu_pack_gbs(n_slabs=1 << 15, pool_slabs=1 << 16):
    """The CPU form of the evict pack: gather n_slabs random 8 KiB slabs of a
    host pool (512 MiB) into a pinned buffer with numpy, one thread; GB/s
    moved (read + written), best of three."""
    import numpy as np
    import torch
    slab = WL["tpb"] * WL["D"] * 4
    rng = np.random.default_rng(1)
    pool = np.full((pool_slabs, slab), 7, dtype=np.uint8)
    dst = torch.zeros(n_slabs, slab, dtype=torch.uint8).pin_memory().numpy()
    idx = np.sort(rng.choice(pool_slabs, n_slabs, replace=False))
    best = float("inf")
    for _ in range(3):
        t0 = time.perf_counter()
        dst[:] = pool[idx]
        best = min(best, time.perf_counter() - t0)
    return round(2 * n_slabs * slab / best / 1e9, 2)


def run_reference(args, rank, world):
    if rank != 0:
        return
    from oracle import oracle as O
    if not O.ref_available():
        print(json.dumps({"impl": "reference", "unavailable":
                          "oracle/_ref was not built (reference sources absent at build time)"}))
        return
    import torch
    torch.cuda.set_device(0)
    threads = max(1, min(host_threads(), WL["B"]))
    m = _reference_sample(steps=max(1, args.steps), warm=min(args.warmup, 1), threads=threads)
    v = round(m["migrated"] / m["step_s"], 1)
    line = {"impl": "reference", "metric": METRIC, "value": v, "unit": "blocks/s",
            "n_gpus": 1, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(m["step_s"] * 1e3, 3), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32+bf16",
            "data": "synthetic (seeded)", "config": {"workload": WL["name"],
                                                     "sample_requests": threads},
            "cpu_baseline": {"value": v, "unit": "blocks/s", "cores": threads,
                             "kind": "reference",
                             "sample": f"{threads} of {WL['B']} requests x 28 layers x 4 KV "
                                       f"heads x 512 blocks ({int(m['blocks'])} blocks), one "
                                       f"request per host thread; scheduler on one thread"},
            "e2e": {"value": v, "unit": "blocks/s", "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0},
            "phases_s": {k: round(v_, 6) for k, v_ in m.items() if k.endswith("_s")}}
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-sharded", action="store_true",
                    help="skip the KV-head-sharded Llama-3-8B-shaped pool")
    ap.add_argument("--sharded-requests", type=int, default=SH["B"],
                    help="requests of the sharded pool (the same at every N)")
    ap.add_argument("--no-three-tier", action="store_true",
                    help="skip the Llama-3-70B-shaped three-tier pool")
    ap.add_argument("--three-tier-requests", type=int, default=TT["B"],
                    help="requests of the three-tier pool (the same at every N)")
    ap.add_argument("--no-cpu-step", action="store_true",
                    help="skip the one-request CPU-runnable step (one GPU only)")
    ap.add_argument("--no-multiplexed", action="store_true",
                    help="skip the Mistral-7B-shaped time-multiplexed pool")
    ap.add_argument("--multiplexed-requests", type=int, default=MX["B"],
                    help="requests of the time-multiplexed pool (the same at every N)")
    ap.add_argument("--requests", type=int, default=WL["B"],
                    help="requests per GPU (32 = the benchmark workload; smaller "
                         "values only for profiling captures)")
    args = ap.parse_args()
    WL["B"] = args.requests
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank, world)
    else:
        run_ours(args, rank, world, local_rank)


if __name__ == "__main__":
    main()
