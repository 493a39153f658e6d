#!/usr/bin/env python
"""Benchmark of the attention hot path on synthetic data.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--repeats R]
    python bench.py --impl reference [...]        # the CPU port of the reference's host attention
    python bench.py --impl reference-gpu          # the reference's own kernels recompiled for sm_100a

The headline workload (`value`, `roofline`, `e2e` of the printed line, at every N) is the
131K-context turbo3 decode: 2 slots x 1 query token, GQA 24/4, head_dim 256, 131072 turbo3 rows
per slot per GPU (K/V drawn N(0,1) through fp16 with 2 % of the (kv head, dim) channels scaled
x8, encoded by the engine's turbo3 store). With N > 1 ranks the KV sequence is split: every
rank holds one 131072-row shard of each slot (context N x 131072, weak scaling), computes
partials over it, and the partials meet through peer-memory mailboxes (or NCCL) and are merged.

The same line carries a `configs` object with the other named workloads, each measured the
same way and checked against the CPU oracle: `c1` (fp16, 4096 rows), `c2` (fp8 verify, 6 lanes x
32768 rows) and `c4` (prefill, TFLOP/s) at N = 1; `c5` (turbo3 verify, 8 slots x 6 lanes x
262144 rows, the rows SPLIT over the ranks: strong scaling) at every N.

One "step" = one pass of attention over one set of resident KV caches. The step rotates over
several distinct cache copies whose total exceeds twice the L2 (or the caches of one step
exceed the L2 several times over), so every timed read comes from HBM. A timed region is K
steps between two CUDA events, bracketed by barrier + synchronize; it is repeated R times and
the MEDIAN region is reported (max over ranks per region), with the spread beside it.
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
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

N_Q, N_KV, HD, GQA = 24, 4, 256, 6
Q_STRIDE = 2 * HD
SCALE = 1.0 / 16.0
KV_F16, KV_FP8, KV_T3 = 0, 1, 2
ROW_BYTES = {KV_F16: 2048, KV_FP8: 1024, KV_T3: 400}
KIND_NAME = {KV_F16: "fp16", KV_FP8: "fp8-e4m3", KV_T3: "turbo3"}
# name -> (kvk, slots, lanes, context rows per slot, outlier fraction, rows split over ranks)
DECODE = {"c1": (KV_F16, 1, 1, 4096, 0.0, False), "c2": (KV_FP8, 1, 6, 32768, 0.0, False),
          "c3": (KV_T3, 2, 1, 131072, 0.02, False), "c5": (KV_T3, 8, 6, 262144, 0.02, True),
          # c5's kernel at a size a profiler capture can hold (2 slots x 65536 rows): only ever
          # run as `--workload c5s`, never part of the default line
          "c5s": (KV_T3, 2, 6, 65536, 0.02, False)}
PREFILL = {"prefix": 8192, "new": 16384, "chunk": 2048}
METRIC = "decode/verify attn KV GB/s (frac of HBM peak) @131K ctx"
PREFILL_METRIC = "prefill attn TFLOP/s"
L2_BYTES = 126 * 2**20
# dram__bytes_read.sum + dram__bytes_write.sum per launch of the dominant kernel, from the ncu
# captures summarised under profiles/ (None where no capture exists for the workload)
NCU_TRAFFIC = {"c3": 213.8e6, "c2": 68.7e6}
BAR = "|got - ref| <= 2e-3 + 1e-3*|ref|"


def peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    try:
        d = json.loads(p.read_text())
        return {"hbm": float(d["hbm_gbs"]), "burst": float(d["bf16_tflops"]),
                "sustained": float(d["bf16_tflops_sustained"]), "source": "measured (MEASURED_PEAKS.json)"}
    except Exception:
        return {"hbm": 6650.0, "burst": 1590.0, "sustained": 1400.0, "source": "fallback"}


def workload_config(name: str, world: int) -> dict:
    """The workload as both arms describe it (nothing about how an arm runs it)."""
    if name == "c4":
        return {"workload": "c4", "kv_kind": "fp16 cache, bf16-rounded values", "heads": "24q/4kv",
                "head_dim": HD, **PREFILL, "parallelism": "single gpu",
                "l2_policy": "Q + KV + out of a step = 1.3 GB > L2"}
    kvk, slots, lanes, rows, outl, split = DECODE[name]
    total = rows if split else rows * world
    per_gpu = -(-(-(-total // 64)) // world) * 64 if split else rows
    step_bytes = slots * min(per_gpu, total) * ROW_BYTES[kvk] * 2
    copies = n_copies(step_bytes)
    return {"workload": name, "kv_kind": KIND_NAME[kvk], "slots": slots, "lanes": lanes,
            "context_rows_per_slot": total, "rows_per_gpu_per_slot": min(per_gpu, total),
            "heads": "24q/4kv", "head_dim": HD,
            "generator": "N(0,1) through fp16" + (f", {outl:.0%} of channels x8" if outl else "") +
                         (", per-head absmax e4m3 scales" if kvk == KV_FP8 else ""),
            "parallelism": f"kv-split x{world}" if world > 1 else "single gpu",
            "l2_policy": f"inputs rotate over {copies} cache copies "
                         f"({copies * step_bytes / 2**20:.0f} MiB > 2 x L2)" if copies > 1 else
                         f"one step reads {step_bytes / 2**20:.0f} MiB > 4 x L2"}


def n_copies(step_bytes: int) -> int:
    if step_bytes >= 4 * L2_BYTES:
        return 1
    return min(24, max(2, -(-2 * L2_BYTES // step_bytes) + 1))


class ClockSampler:
    """Samples SM clocks and throttle reasons with nvidia-smi while the timed region runs."""

    FIELDS = ("clocks.sm,clocks.max.sm,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.samples = []
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except Exception:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.samples.append(line.strip())

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        clocks, maxes, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for s in self.samples:
            f = [x.strip() for x in s.split(",")]
            if len(f) < 6:
                continue
            try:
                clocks.append(float(f[0]))
                maxes.append(float(f[1]))
            except ValueError:
                continue
            for n, v in zip(names, f[2:6]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        clocks.sort()
        # under load = the upper half of the samples (idle samples sit at the floor clock)
        load = clocks[len(clocks) // 2:] if clocks else []
        med = load[len(load) // 2] if load else None
        return {"sm_mhz": med, "sm_max_mhz": max(maxes) if maxes else None,
                "reasons": sorted(reasons), "samples": len(clocks)}


def tolerance_ok(got, ref) -> tuple[bool, float]:
    import numpy as np
    err = np.abs(np.asarray(got, dtype=np.float64) - np.asarray(ref, dtype=np.float64))
    excess = float((err - (2e-3 + 1e-3 * np.abs(ref))).max())
    return excess <= 0.0, excess


# ---- our arm: decode / verify workloads -----------------------------------------------------

class DecodeRun:
    """One decode / verify workload resident on this rank: caches, the step, its timings."""

    def __init__(self, name, args, world, rank, dev):
        import torch
        import torch.distributed as dist

        import q27_b200 as Q
        from q27_b200 import dist as qd
        from q27_b200 import workloads as W
        self.torch, self.dist, self.Q, self.qd, self.W = torch, dist, Q, qd, W
        self.name, self.args, self.world, self.rank, self.dev = name, args, world, rank, dev
        kvk, nslots, lanes, rows, outl, split = DECODE[name]
        self.kvk, self.nslots, self.lanes = kvk, nslots, lanes
        if split:                        # strong scaling: the context is divided over the ranks
            self.rows_total = rows
            self.lo, self.hi = qd.shard_ranges(rows, world)[rank]
            self.scaling = "strong"
        else:                            # weak scaling: every rank holds `rows` rows
            self.rows_total = rows * world
            self.lo, self.hi = rank * rows, (rank + 1) * rows
            self.scaling = "weak"
        self.local_rows = self.hi - self.lo
        self.step_bytes_rank = nslots * self.local_rows * ROW_BYTES[kvk] * 2   # K+V, counted once
        self.copies = copies = n_copies(max(self.step_bytes_rank, 1))
        self.caches = [[W.make_cache(kvk, self.local_rows, 100 * c + s, outl, dev, first_row=self.lo)
                        for s in range(nslots)] for c in range(copies)]
        q0 = W.make_queries(nslots, lanes, seed=4242)
        pos_vals = torch.tensor([[self.rows_total - lanes + t for t in range(lanes)]
                                 for _ in range(nslots)], dtype=torch.int32)
        # A step's inputs (Q lanes, then positions) sit in ONE pinned host block and one device
        # block per cache copy, so the end-to-end step moves them with a single copy. fp8: the K
        # side's per-head scale of that copy's cache is folded into its Q (the cache is scale-free).
        self.q_bytes = q0.numel() * 4
        self.in_host, self.in_dev, self.q_dev, self.pos_dev, self.q_host = [], [], [], [], []
        for c in range(copies):
            qc = q0
            if kvk == KV_FP8:
                qc = torch.stack([W.fold_k_scale(q0[s], self.caches[c][s].k_scale.cpu()) for s in range(nslots)])
            h = torch.empty(self.q_bytes + pos_vals.numel() * 4, dtype=torch.uint8).pin_memory()
            h[:self.q_bytes].view(torch.float32).copy_(qc.reshape(-1))
            h[self.q_bytes:].view(torch.int32).copy_(pos_vals.view(-1))
            d = torch.empty_like(h, device=dev)
            d.copy_(h)
            self.in_host.append(h)
            self.in_dev.append(d)
            self.q_host.append(h[:self.q_bytes].view(torch.float32).view(nslots, lanes, N_Q * Q_STRIDE))
            self.q_dev.append(d[:self.q_bytes].view(torch.float32).view(nslots, lanes, N_Q * Q_STRIDE))
            self.pos_dev.append(d[self.q_bytes:].view(torch.int32).view(nslots, lanes))
        self.pos_host = pos_vals
        self.out_dev = torch.zeros((nslots, lanes, N_Q * HD), device=dev)
        self.out_host = torch.zeros((nslots, lanes, N_Q * HD)).pin_memory()
        self.scratch = [torch.empty(Q.decode_scratch_floats(lanes), device=dev) for _ in range(nslots)]
        self.merged = torch.zeros((nslots * lanes * N_Q, HD), device=dev)
        self.boxes = self.ex = None
        if world > 1 and args.exchange == "peer":
            try:
                self.boxes = qd.PeerMailboxes(nslots, lanes, N_Q, device_epoch=not args.no_graph)
            except RuntimeError as e:     # raised on every rank together: fall back together
                if rank == 0:
                    print(f"bench: {e}; using the NCCL exchange", file=sys.stderr)
        if world > 1:
            self.ex = qd.PartialExchange.create(nslots, lanes, N_Q, world, dev)
        self.slot_sets = [self._slots(c) for c in range(copies)]
        # argument blocks marshalled once, as an engine that replays the same pointers does
        self.calls = [Q.BatchedDecode(sl, Q_STRIDE, N_Q, N_KV, HD, SCALE, kvk=kvk) for sl in self.slot_sets]
        self.marshalled = [Q.marshal_slots(sl) for sl in self.slot_sets]
        self.use_graph = not args.no_graph and (world == 1 or self.boxes is not None)
        # Across ranks a step's merge waits (bounded, about half a second) for every rank's push:
        # the ranks enter each group of steps together, whatever their host-side set-up took.
        self.barrier()
        self.launches_per_step = self._count_launches()
        self.barrier()
        self.round_graph = self._graph(lambda: [self.step(c) for c in range(copies)]) if self.use_graph else None
        self.e2e_graphs = None
        if self.use_graph:
            self.e2e_graphs = []
            for c in range(copies):
                self.barrier()
                self.e2e_graphs.append(self._graph(lambda c=c: self._e2e_body(c)))
        self.barrier()

    def _slots(self, c):
        Q = self.Q
        return [Q.SlotArgs(self.caches[c][s].ktab, self.caches[c][s].vtab,
                           [self.q_dev[c][s, t] for t in range(self.lanes)],
                           [self.pos_dev[c][s, t:t + 1] for t in range(self.lanes)],
                           [self.out_dev[s, t] for t in range(self.lanes)], self.scratch[s],
                           row_base=self.lo if self.world > 1 else 0,
                           row_count=self.local_rows if self.world > 1 else 2**31 - 1)
                for s in range(self.nslots)]

    def step(self, i, exchange=None):
        c = i % self.copies
        how = exchange or ("peer" if self.boxes is not None else "nccl")
        if self.world == 1:
            self.calls[c]()
        elif how == "peer":
            self.boxes.decode(self.marshalled[c], self.merged, Q_STRIDE, N_KV, SCALE, self.kvk)
        else:
            self.qd.sharded_decode(self.slot_sets[c], self.ex, self.merged, Q_STRIDE, N_KV, SCALE, self.kvk)

    def result(self):
        """[nslots, lanes, 6144] of the last step, on the device."""
        return self.merged.view(self.nslots, self.lanes, N_Q * HD) if self.world > 1 else self.out_dev

    def barrier(self):
        self.torch.cuda.synchronize()
        if self.world > 1:
            self.dist.barrier()
            self.torch.cuda.synchronize()

    def _count_launches(self) -> int:
        """Kernels of this library in one step, counted by the library itself."""
        self.step(0)
        self.torch.cuda.synchronize()
        n0 = self.Q.launch_count()
        self.step(0)
        self.torch.cuda.synchronize()
        return self.Q.launch_count() - n0

    def _graph(self, fn):
        # One CUDA graph holds a round of `copies` consecutive steps (every launch of the library
        # is capturable and, with device-counted exchange epochs, has constant arguments), as the
        # engine this path drops into replays its decode step from a graph.
        torch = self.torch
        side = torch.cuda.Stream()
        side.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(side):
            fn()
        torch.cuda.current_stream().wait_stream(side)
        self.barrier()               # the warm-up steps have run on every rank before the capture
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            fn()
        return graph

    def run_steps(self, n):
        i = 0
        while n > 0:
            if self.round_graph is not None and i % self.copies == 0 and n >= self.copies:
                self.round_graph.replay()
                i, n = i + self.copies, n - self.copies
            else:
                self.step(i)
                i, n = i + 1, n - 1

    def _max_over_ranks(self, values):
        if self.world == 1:
            return list(values)
        t = self.torch.tensor(list(values), device=self.dev, dtype=self.torch.float64)
        self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX)
        return t.tolist()

    def time_device(self, steps, repeats):
        """ms per step of `repeats` timed regions of `steps` steps each (max over ranks)."""
        torch = self.torch
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        out = []
        for _ in range(repeats):
            self.barrier()
            e0.record()
            self.run_steps(steps)
            e1.record()
            self.barrier()
            out.append(e0.elapsed_time(e1) / steps)
        return self._max_over_ranks(out)

    def time_call_patterns(self, steps) -> dict:
        """The step launched directly (no graph) in two ways: the batched entry with all slots
        in one call, and the way the reference's engine would call a drop-in today -- one
        single-slot `attn_decode3` per request, each on its own stream, running concurrently.
        ms per step, single GPU."""
        torch, Q = self.torch, self.Q
        main = torch.cuda.current_stream()
        streams = [torch.cuda.Stream() for _ in range(self.nslots)]
        fork, joins = torch.cuda.Event(), [torch.cuda.Event() for _ in range(self.nslots)]

        def batched(i):
            self.calls[i % self.copies]()

        def per_request(i):
            sl = self.slot_sets[i % self.copies]
            fork.record(main)
            for s, st in enumerate(streams):
                st.wait_event(fork)
                with torch.cuda.stream(st):
                    a = sl[s]
                    Q.attn_decode3(a.q_lanes, Q_STRIDE, a.ktab, a.vtab, a.out_lanes, a.scratch, a.pos_lanes,
                                   0, N_Q, N_KV, HD, SCALE, st=st, ntok=self.lanes, kvk=self.kvk)
                joins[s].record(st)
            for j in joins:
                main.wait_event(j)

        out = {}
        for name, fn in (("batched_direct_ms", batched), ("one_call_per_request_on_own_streams_ms", per_request)):
            for i in range(6):
                fn(i)
            torch.cuda.synchronize()
            ms = []
            for _ in range(15):
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                for i in range(steps):
                    fn(i)
                e1.record()
                torch.cuda.synchronize()
                ms.append(e0.elapsed_time(e1) / steps)
            out[name] = round(statistics.median(ms), 5)
        return out

    def time_kernel(self, steps):
        """Mean duration of the dominant (split-KV partial) kernel, bracketed by events that the
        library records on the launch stream right around it."""
        torch, lib = self.torch, self.Q._lib.lib()
        k0 = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
        k1 = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
        for i in range(steps):
            k0[i].record()
            k1[i].record()                          # materialise the handles; re-recorded below
            lib.q27_set_kernel_events(k0[i].cuda_event, k1[i].cuda_event)
            self.step(i)
        lib.q27_set_kernel_events(None, None)
        self.barrier()
        ms = sorted(a.elapsed_time(b) for a, b in zip(k0, k1))
        return sum(ms) / len(ms)

    def _e2e_body(self, c):
        self.in_dev[c].copy_(self.in_host[c], non_blocking=True)
        self.step(c)
        self.out_host.copy_(self.result(), non_blocking=True)

    def time_e2e(self, steps, warmup):
        """Seconds per step through the public call with HOST buffers: the step's inputs come
        from pinned host memory, its output rows go back, one stream sync per step."""
        torch = self.torch

        def one(i):
            if self.e2e_graphs is not None:
                self.e2e_graphs[i % self.copies].replay()
            else:
                self._e2e_body(i % self.copies)
            torch.cuda.current_stream().synchronize()
        for i in range(warmup):
            one(i)
        self.barrier()
        t0 = time.perf_counter()
        for i in range(steps):
            one(i)
        self.barrier()
        return self._max_over_ranks([(time.perf_counter() - t0) / steps])[0]

    # ---- checks --------------------------------------------------------------------------
    def check(self, oracle) -> str:
        """Before anything is timed: the result of one step against the CPU oracle (slot 0, all
        lanes, the whole context) and, across GPUs, the peer-memory exchange against NCCL."""
        torch, dist = self.torch, self.dist
        notes = []
        if self.world > 1 and self.boxes is not None:
            self.step(0, "nccl")
            torch.cuda.synchronize()
            via_nccl = self.merged.clone()
            self.step(0, "peer")
            torch.cuda.synchronize()
            same = torch.equal(via_nccl.view(torch.int32), self.merged.view(torch.int32))
            flags = [same] * self.world
            dist.all_gather_object(flags, same)
            if not all(flags):
                raise SystemExit(f"{self.name}: peer-memory and NCCL exchanges disagree")
            notes.append("peer-memory exchange bitwise equal to the NCCL exchange on every rank")
        else:
            self.step(0)
            torch.cuda.synchronize()
        if oracle is None:
            return "; ".join(notes + ["oracle check skipped (--no-cpu)"])
        got = self.result()[0].clone()
        cache = self.caches[0][0]
        rb = ROW_BYTES[self.kvk]
        ks = cache.kstore[: self.local_rows * rb]
        vs = cache.vstore[: self.local_rows * rb]
        if self.world > 1:                 # slot 0's shards meet on rank 0 (rows are in rank order)
            parts = []
            for side in (ks, vs):
                sizes = [0] * self.world
                dist.all_gather_object(sizes, side.numel())
                pad = torch.zeros(max(sizes), dtype=torch.uint8, device=self.dev)
                pad[: side.numel()] = side
                gl = [torch.empty_like(pad) for _ in range(self.world)] if self.rank == 0 else None
                dist.gather(pad, gl, dst=0)
                if self.rank == 0:
                    parts.append(torch.cat([g[:n] for g, n in zip(gl, sizes)]).cpu())
            if self.rank != 0:
                return ""
            ks, vs = parts
        k = ks.cpu().numpy().reshape(-1, rb)
        v = vs.cpu().numpy().reshape(-1, rb)
        q = self.q_host[0][0].numpy().reshape(self.lanes, N_Q, Q_STRIDE)
        ref = oracle.attn_decode(q, k, v, self.kvk, self.pos_host[0].tolist())
        g = got.cpu()
        if self.kvk == KV_FP8:             # parity is judged on the real-valued outputs
            g = self.W.apply_v_scale(g, cache.v_scale.cpu())
            ref = self.W.apply_v_scale(torch.from_numpy(ref), cache.v_scale.cpu()).numpy()
        ok, excess = tolerance_ok(g.numpy(), ref)
        if not ok:
            raise SystemExit(f"{self.name}: GPU result disagrees with the CPU oracle (excess {excess:.3e})")
        notes.append(f"slot 0 ({self.lanes} lanes x {k.shape[0]} rows) equals the CPU oracle within {BAR}")
        return "; ".join(notes)

    def close(self):
        if self.boxes is not None:
            self.boxes.close()
        self.round_graph = self.e2e_graphs = None
        self.caches = self.calls = self.slot_sets = None
        self.torch.cuda.empty_cache()


def measure_decode(run: DecodeRun, args, oracle, repeats) -> dict:
    checked = run.check(oracle)
    if run.world > 1 and run.rank == 0 and not checked:
        checked = "checked on rank 0"
    # rank 0 has just spent seconds in the CPU oracle: nobody launches a step (whose merge waits,
    # bounded, for every rank's push) before everybody is back
    run.barrier()
    run.run_steps(args.warmup)
    ms_list = run.time_device(args.steps, repeats)
    kernel_ms = run.time_kernel(args.steps)
    e2e_s = run.time_e2e(args.steps, args.warmup)
    ms = statistics.median(ms_list)
    total_bytes = run.step_bytes_rank * run.world if run.scaling == "weak" else \
        run.nslots * run.rows_total * ROW_BYTES[run.kvk] * 2
    pk = peaks()
    achieved = run.step_bytes_rank / (kernel_ms * 1e-3) / 1e9
    how = ("none" if run.world == 1 else "peer-memory mailboxes (P2P stores + flags, no collective)"
           if run.boxes is not None else "nccl all-gather")
    return {
        "value": round(total_bytes / (ms * 1e-3) / 1e9, 2), "unit": "GB/s",
        "ms_per_step": round(ms, 5), "ms_per_step_min": round(min(ms_list), 5),
        "ms_per_step_max": round(max(ms_list), 5), "repeats": repeats, "scaling": run.scaling,
        "algorithmic_bytes_per_step": total_bytes,
        "kernel_ms": round(kernel_ms, 5),
        "kernel": ("k_verify_umma (tcgen05, split-KV partials)" if run.lanes >= 2
                   else "k_decode_mma (split-KV partials" +
                   (" + merge in the same launch)" if run.launches_per_step == 1 else ")")),
        "algorithmic_bytes_per_launch": run.step_bytes_rank,
        "achieved": round(achieved, 1), "peak": pk["hbm"], "frac": round(achieved / pk["hbm"], 4),
        "frac_of_nominal_8TBps": round(achieved / 8000.0, 4),
        "step_frac": round(run.step_bytes_rank / (ms * 1e-3) / 1e9 / pk["hbm"], 4),
        "e2e": {"value": round(total_bytes / e2e_s / 1e9, 2), "unit": "GB/s",
                "h2d_bytes_per_step": int(run.in_host[0].numel()),
                "d2h_bytes_per_step": int(run.out_host.numel() * 4)},
        "gpu_launches_per_step": run.launches_per_step,
        "launch": (f"cuda graph per round of {run.copies} steps" if run.use_graph else "direct launches"),
        "exchange": how, "checked": checked,
        "config": workload_config(run.name, run.world),
    }


# ---- our arm: the prefill workload ---------------------------------------------------------

def measure_prefill(args, oracle, repeats) -> dict:
    """One step = the 8 chunks of 2048 new tokens over the 8192-row prefix (store the chunk's
    K/V rows, then causal attention over prefix + chunk)."""
    import numpy as np
    import torch

    import q27_b200 as Q
    from q27_b200 import workloads as W
    dev = torch.device("cuda", torch.cuda.current_device())
    PREFIX, NEW, CH = PREFILL["prefix"], PREFILL["new"], PREFILL["chunk"]
    rows = PREFIX + NEW
    g = torch.Generator(device=dev)
    g.manual_seed(7)
    rb = ROW_BYTES[KV_F16]
    stores = [torch.empty(((rows + 63) // 64) * 64 * rb, dtype=torch.uint8, device=dev) for _ in range(2)]
    ktab, vtab = Q.mk_tab(stores[0], rb, rows), Q.mk_tab(stores[1], rb, rows)
    for r0 in range(0, PREFIX, 4096):
        Q.kv_store_T(W.bf16_values((4096, N_KV * HD), g, dev), W.bf16_values((4096, N_KV * HD), g, dev),
                     ktab, vtab, r0, N_KV * HD, 4096)
    qT = W.bf16_values((NEW, N_Q * Q_STRIDE), g, dev)
    kT = W.bf16_values((NEW, N_KV * HD), g, dev)
    vT = W.bf16_values((NEW, N_KV * HD), g, dev)
    outT = torch.zeros((NEW, N_Q * HD), device=dev)
    part = torch.empty(Q.prefill_part_floats(CH), device=dev)
    out_host = torch.zeros((CH, N_Q * HD)).pin_memory()
    q_host = qT[:CH].cpu().pin_memory()

    def attn(c):
        sl = slice(c * CH, (c + 1) * CH)
        Q.attn_prefill_T(qT[sl], Q_STRIDE, N_Q * Q_STRIDE, ktab, vtab, outT[sl], N_Q * HD, part,
                         PREFIX + c * CH, 0, CH, N_Q, N_KV, HD, SCALE, kvk=KV_F16)

    def step(e2e=False):
        for c in range(NEW // CH):
            sl = slice(c * CH, (c + 1) * CH)
            if e2e:   # the chunk's Q rows come from the host, its output rows go back
                qT[sl].copy_(q_host, non_blocking=True)
            Q.kv_store_T(kT[sl], vT[sl], ktab, vtab, PREFIX + c * CH, N_KV * HD, CH)
            attn(c)
            if e2e:
                out_host.copy_(outT[sl], non_blocking=True)
        if e2e:
            torch.cuda.current_stream().synchronize()

    n0 = Q.launch_count()
    step()
    torch.cuda.synchronize()
    launches = Q.launch_count() - n0
    checked = "oracle check skipped (--no-cpu)"
    if oracle is not None:    # query rows 0..63 of the first chunk against the CPU oracle
        kh = stores[0][: (PREFIX + CH) * rb].cpu().numpy().reshape(-1, rb)
        vh = stores[1][: (PREFIX + CH) * rb].cpu().numpy().reshape(-1, rb)
        ref = oracle.attn_prefill(qT[:CH].cpu().numpy().reshape(CH, N_Q, Q_STRIDE), kh, vh, KV_F16, PREFIX, 0, 64)
        ok, excess = tolerance_ok(outT[:64].cpu().numpy(), ref[:64])
        if not ok:
            raise SystemExit(f"c4: GPU result disagrees with the CPU oracle (excess {excess:.3e})")
        checked = f"query rows 0..63 of the first chunk equal the CPU oracle within {BAR}"
    pairs = sum(CH * (PREFIX + CH * c) + CH * (CH + 1) // 2 for c in range(NEW // CH))
    flops = pairs * N_Q * 4 * HD
    def kernels_alone():
        ka = [torch.cuda.Event(enable_timing=True) for _ in range(2 * (NEW // CH))]
        for c in range(NEW // CH):
            ka[2 * c].record()
            attn(c)
            ka[2 * c + 1].record()
        torch.cuda.synchronize()
        return sum(ka[2 * c].elapsed_time(ka[2 * c + 1]) for c in range(NEW // CH))

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    # the attention kernels alone, right after the warm-up: a few milliseconds of work, the
    # conditions of the burst figure of the measured cuBLAS peak
    kernel_ms = min(kernels_alone() for _ in range(2))
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ms_list = []
    steps = max(1, min(args.steps, 10))
    for _ in range(repeats):
        torch.cuda.synchronize()
        e0.record()
        for _ in range(steps):
            step()
        e1.record()
        torch.cuda.synchronize()
        ms_list.append(e0.elapsed_time(e1) / steps)
    ms = statistics.median(ms_list)
    # the same after the long loop (power-capped clocks): against the sustained peak
    kernel_ms_sustained = kernels_alone()
    for _ in range(2):
        step(e2e=True)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(steps):
        step(e2e=True)
    torch.cuda.synchronize()
    e2e_s = (time.perf_counter() - t0) / steps
    pk = peaks()
    achieved = flops / (kernel_ms * 1e-3) / 1e12
    return {
        "metric": PREFILL_METRIC, "value": round(flops / (ms * 1e-3) / 1e12, 2), "unit": "TFLOP/s",
        "ms_per_step": round(ms, 4), "ms_per_step_min": round(min(ms_list), 4),
        "ms_per_step_max": round(max(ms_list), 4), "repeats": repeats, "steps_per_region": steps,
        "algorithmic_flops_per_step": flops, "kernel_ms": round(kernel_ms, 4),
        "kernel": "k_prefill_umma (tcgen05)", "achieved": round(achieved, 2),
        # kernel_ms / achieved / frac: the eight attention kernels of a step timed alone right
        # after the warm-up, against the burst figure of the measured cuBLAS bf16 peak; the
        # *_sustained pair: the same kernels after the long timed loop, against the sustained one
        "peak": pk["burst"], "frac": round(achieved / pk["burst"], 4),
        "kernel_ms_sustained": round(kernel_ms_sustained, 4),
        "achieved_sustained": round(flops / (kernel_ms_sustained * 1e-3) / 1e12, 2),
        "frac_sustained": round(flops / (kernel_ms_sustained * 1e-3) / 1e12 / pk["sustained"], 4),
        "frac_of_nominal_2250TF": round(achieved / 2250.0, 4),
        "e2e": {"value": round(flops / e2e_s / 1e12, 2), "unit": "TFLOP/s",
                "h2d_bytes_per_step": int(q_host.numel() * 4 * (NEW // CH)),
                "d2h_bytes_per_step": int(out_host.numel() * 4 * (NEW // CH))},
        "gpu_launches_per_step": launches, "checked": checked, "dtype": "f16",
        "config": workload_config("c4", 1),
    }


def run_ours(args):
    import torch
    import torch.distributed as dist

    import q27_b200 as Q

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus and world == 1 and args.gpus > 1:
        raise SystemExit("launch N>1 with torch.distributed.run (one rank per GPU)")
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev)
    if Q._lib.lib().q27_device_arch() != 1000:
        raise SystemExit("the engine is built for sm_100a only")
    oracle = None
    if not args.no_cpu:
        from tests.oracle_lib import Oracle
        oracle = Oracle()

    main_name = args.workload or "c3"
    if main_name == "c4":
        line = measure_prefill(args, oracle, max(3, args.repeats // 5))
        line.update({"n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "higher_is_better": True,
                     "scaling": "weak", "vs_baseline": None, "data": "synthetic",
                     "gpu_launches": line["gpu_launches_per_step"] * args.steps,
                     "roofline": {"bound": "tensor", "achieved": line["achieved"], "peak": line["peak"],
                                  "unit": "TFLOP/s", "frac": line["frac"], "traffic": None}})
        if rank == 0:
            print(json.dumps(line), flush=True)
        return

    run = DecodeRun(main_name, args, world, rank, dev)
    sampler = ClockSampler(local_rank)
    if rank == 0:
        sampler.start()
        time.sleep(0.15)
    m = measure_decode(run, args, oracle, args.repeats)
    clocks = sampler.stop() if rank == 0 else None
    patterns = run.time_call_patterns(args.steps) if world == 1 and run.nslots > 1 else None
    cpu_base = None
    if rank == 0 and world == 1 and oracle is not None and main_name == "c3":
        cpu_base = cpu_baseline(run, oracle)
    run.close()

    configs = {}
    if args.workload is None:
        others = ["c1", "c2", "c5"] if world == 1 else ["c5"]
        for name in others:
            r = DecodeRun(name, args, world, rank, dev)
            configs[name] = measure_decode(r, args, oracle, max(5, args.repeats // (5 if name == "c5" else 1)))
            r.close()
        if world == 1:
            configs["c4"] = measure_prefill(args, oracle, max(3, args.repeats // 5))

    flag = C.c_int(0)
    Q._lib.lib().q27_wait_timeout_flag(C.byref(flag))
    if flag.value:
        raise SystemExit("a bounded device wait timed out during the run: numbers are invalid")

    kvk = run.kvk
    line = {
        "metric": METRIC, "value": m["value"], "unit": "GB/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": m["ms_per_step"],
        "ms_per_step_min": m["ms_per_step_min"], "ms_per_step_max": m["ms_per_step_max"],
        "repeats": m["repeats"], "higher_is_better": True, "scaling": m["scaling"], "vs_baseline": None,
        "dtype": "u8" if kvk != KV_F16 else "f16", "data": "synthetic",
        "config": m["config"],
        "run": {"launch": m["launch"], "exchange": m["exchange"], "checked": m["checked"],
                **({"call_patterns": patterns} if patterns else {})},
        "e2e": dict(m["e2e"], note="Q lanes + positions in from pinned host memory, outputs back, one "
                                   "stream sync per step; the KV cache is engine state resident in HBM"),
        "gpu_launches": m["gpu_launches_per_step"] * args.steps,
        "clocks": clocks,
        "roofline": {"bound": "hbm", "achieved": m["achieved"], "peak": m["peak"], "unit": "GB/s",
                     "frac": m["frac"], "traffic": NCU_TRAFFIC.get(main_name),
                     "peak_source": f"{peaks()['source']}: copy bandwidth",
                     "kernel": m["kernel"], "kernel_ms": m["kernel_ms"],
                     "algorithmic_bytes_per_launch": m["algorithmic_bytes_per_launch"],
                     "frac_of_nominal_8TBps": m["frac_of_nominal_8TBps"]},
    }
    if cpu_base is not None:
        line["cpu_baseline"] = cpu_base
    if configs:
        line["configs"] = configs
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


def cpu_baseline(run: DecodeRun, oracle) -> dict:
    """The CPU oracle (a port of the reference's scalar host attention), timed on the host
    cores over the whole workload once: every slot, every row."""
    cores = os.cpu_count() or 1
    rb = ROW_BYTES[run.kvk]
    secs = 0.0
    for s in range(run.nslots):
        k, v = run.caches[0][s].host_rows()
        q = run.q_host[0][s].numpy().reshape(run.lanes, N_Q, Q_STRIDE)
        t0 = time.perf_counter()
        oracle.attn_decode(q, k, v, run.kvk, run.pos_host[s].tolist(), nthreads=cores)
        secs += time.perf_counter() - t0
    nbytes = run.nslots * run.local_rows * rb * 2
    return {"value": round(nbytes / secs / 1e9, 4), "unit": "GB/s", "cores": cores, "kind": "port",
            "sample": f"the whole step once: {run.nslots} slots x {run.lanes} lanes x {run.local_rows} "
                      f"rows, {secs:.2f} s (OpenMP over lane x head, {cores} threads)"}


# ---- the reference arm: the reference's host attention on the host cores ---------------------

def run_reference(args):
    """The CPU restatement of the reference's scalar host attention (its own host_ref lives
    inside a test binary and cannot be built apart), all host threads, on the headline
    workload: same generator, same shapes. Each step is one pass over every slot; at N > 1
    the per-GPU shard (131072 rows per slot) stands for the N-times longer context, because the
    cost is linear in rows and the metric is bytes per second."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    import numpy as np

    from tests.oracle_lib import Oracle
    o = Oracle()
    name = args.workload or "c3"
    if name == "c4":
        print(json.dumps({"impl": "reference", "unavailable": "the reference arm times the decode workloads"}))
        return
    kvk, nslots, lanes, rows, outl, split = DECODE[name]
    world = args.gpus
    cores = os.cpu_count() or 1
    rb = ROW_BYTES[kvk]
    srows = rows if not split else min(rows, 131072)
    # torchrun exports OMP_NUM_THREADS=1: the thread count is passed explicitly everywhere
    kf = o.randn(srows * N_KV * HD, 1, nthreads=cores).reshape(srows, N_KV * HD)
    vf = o.randn(srows * N_KV * HD, 2, nthreads=cores).reshape(srows, N_KV * HD)
    if outl > 0:
        rng = np.random.default_rng(11)
        n = max(1, int(round(outl * N_KV * HD)))
        kf[:, rng.choice(N_KV * HD, n, replace=False)] *= np.float32(8.0)
        vf[:, rng.choice(N_KV * HD, n, replace=False)] *= np.float32(8.0)
    kf = o.to_half_bits(kf).view(np.float16).astype(np.float32)
    vf = o.to_half_bits(vf).view(np.float16).astype(np.float32)
    if kvk == KV_T3:
        k, v = o.t3_quant(kf).reshape(srows, rb), o.t3_quant(vf).reshape(srows, rb)
    elif kvk == KV_FP8:
        k, v = o.to_e4m3(kf * 74.0), o.to_e4m3(vf * 74.0)
    else:
        k, v = o.to_half_bits(kf).view(np.uint8).reshape(srows, rb), \
            o.to_half_bits(vf).view(np.uint8).reshape(srows, rb)
    q = o.randn(lanes * N_Q * Q_STRIDE, 3).reshape(lanes, N_Q, Q_STRIDE)
    pos = [srows - lanes + t for t in range(lanes)]
    for _ in range(max(1, min(args.warmup, 2))):
        o.attn_decode(q, k, v, kvk, pos, nthreads=cores)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        for _s in range(nslots):
            o.attn_decode(q, k, v, kvk, pos, nthreads=cores)
    secs = time.perf_counter() - t0
    sample_bytes = nslots * srows * rb * 2
    value = sample_bytes * args.steps / secs / 1e9
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 4), "unit": "GB/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(secs / args.steps * 1e3, 3), "higher_is_better": True,
        "scaling": "strong" if split else "weak", "vs_baseline": None,
        "dtype": "f64", "data": "synthetic",
        "config": workload_config(name, world),
        "cpu_baseline": {"value": round(value, 4), "unit": "GB/s", "cores": cores, "kind": "port",
                         "sample": f"each step = {nslots} slots x {lanes} lanes x {srows} rows "
                                   f"(one GPU's shard; cost is linear in rows), {cores} threads"},
        "e2e": {"value": round(value, 4), "unit": "GB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
        "gpu_launches": 0,
    }
    print(json.dumps(line), flush=True)


# ---- the reference's own kernels, recompiled for sm_100a, on the same buffers -------------

def run_reference_gpu(args):
    """Times the reference's decode / verify / prefill kernels (oracle/_ref/libq27ref_gpu.so,
    compiled from the reference tree by oracle/Makefile) next to this engine's on identical
    device buffers: same caches, same rotation over cache copies, CUDA events. One GPU."""
    import torch

    import q27_b200 as Q
    from q27_b200 import workloads as W
    so = ROOT / "oracle" / "_ref" / "libq27ref_gpu.so"
    if not so.exists():
        print(json.dumps({"impl": "reference-gpu", "unavailable": f"{so.name} was not built "
                          "(needs the reference tree at build time)"}))
        return
    ref = C.CDLL(str(so))
    vp, i, f = C.c_void_p, C.c_int, C.c_float
    ref.q27ref_attn_decode3.argtypes = [vp, i, vp, vp, vp, vp, vp, i, i, i, f, vp, i, i, i]
    ref.q27ref_attn_decode3.restype = None
    ref.q27ref_attn_prefill_T.argtypes = [vp, i, i, vp, vp, vp, i, vp, i, i, i, i, i, i, f, vp, i]
    ref.q27ref_attn_prefill_T.restype = None
    dev = torch.device("cuda:0")
    torch.cuda.set_device(0)
    st = torch.cuda.current_stream().cuda_stream
    out = {"impl": "reference-gpu", "unit": "ms per step", "n_gpus": 1, "workloads": {}}

    def timeit(fn, steps):
        for s in range(3):
            fn(s)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for s in range(steps):
            fn(s)
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / steps

    for name, fd in (("c3", None), ("c1", None), ("c2", None), ("c2", "mma")):
        kvk, nslots, lanes, rows, outl, _ = DECODE[name]
        if fd:
            os.environ["Q27_FD"] = fd      # the reference reads its dispatch switch at launch
        else:
            os.environ.pop("Q27_FD", None)
        step_bytes = nslots * rows * ROW_BYTES[kvk] * 2
        copies = n_copies(step_bytes)
        caches = [[W.make_cache(kvk, rows, 100 * c + s, outl, dev) for s in range(nslots)] for c in range(copies)]
        q = W.make_queries(nslots, lanes, 4242).to(dev)
        pos = torch.tensor([[rows - lanes + t for t in range(lanes)]] * nslots, dtype=torch.int32, device=dev)
        o = torch.zeros((nslots, lanes, N_Q * HD), device=dev)
        scr = [torch.empty(Q.decode_scratch_floats(lanes), device=dev) for _ in range(nslots)]
        arrs = []
        for s in range(nslots):
            arrs.append(((vp * 16)(*[q[s, t].data_ptr() for t in range(lanes)]),
                         (vp * 16)(*[o[s, t].data_ptr() for t in range(lanes)]),
                         (vp * 16)(*[pos[s, t:t + 1].data_ptr() for t in range(lanes)])))

        def ref_step(it):
            c = it % copies
            for s in range(nslots):     # the reference runs one call per slot (src/conductor.h:681-694)
                qa, oa, pa = arrs[s]
                ref.q27ref_attn_decode3(qa, Q_STRIDE, caches[c][s].ktab.data_ptr(), caches[c][s].vtab.data_ptr(),
                                        oa, scr[s].data_ptr(), pa, N_Q, N_KV, HD, SCALE, st, lanes, kvk, 0)
        calls = [Q.BatchedDecode([Q.SlotArgs(caches[c][s].ktab, caches[c][s].vtab, [q[s, t] for t in range(lanes)],
                                             [pos[s, t:t + 1] for t in range(lanes)],
                                             [o[s, t] for t in range(lanes)], scr[s]) for s in range(nslots)],
                                 Q_STRIDE, N_Q, N_KV, HD, SCALE, kvk=kvk) for c in range(copies)]
        t_ref = timeit(ref_step, args.steps)
        t_ours = timeit(lambda it: calls[it % copies](), args.steps)
        key = name + ("+Q27_FD=mma" if fd else "")
        out["workloads"][key] = {"reference_ms": round(t_ref, 5), "ours_ms": round(t_ours, 5),
                                 "speedup": round(t_ref / t_ours, 2),
                                 "reference_GBps": round(step_bytes / t_ref / 1e6, 1),
                                 "ours_GBps": round(step_bytes / t_ours / 1e6, 1),
                                 "launches": "direct (no graph) on both sides"}
        del caches, calls
        torch.cuda.empty_cache()
    os.environ.pop("Q27_FD", None)

    # prefill: the first and the last 2048-token chunk of the prefill workload
    PREFIX, NEW, CH = PREFILL["prefix"], PREFILL["new"], PREFILL["chunk"]
    rows = PREFIX + NEW
    g = torch.Generator(device=dev)
    g.manual_seed(7)
    rb = ROW_BYTES[KV_F16]
    stores = [torch.empty(((rows + 63) // 64) * 64 * rb, dtype=torch.uint8, device=dev) for _ in range(2)]
    ktab, vtab = Q.mk_tab(stores[0], rb, rows), Q.mk_tab(stores[1], rb, rows)
    for r0 in range(0, rows, 4096):
        Q.kv_store_T(W.bf16_values((4096, N_KV * HD), g, dev), W.bf16_values((4096, N_KV * HD), g, dev),
                     ktab, vtab, r0, N_KV * HD, 4096)
    qT = W.bf16_values((CH, N_Q * Q_STRIDE), g, dev)
    outT = torch.zeros((CH, N_Q * HD), device=dev)
    part = torch.empty(Q.prefill_part_floats(CH), device=dev)
    for base in (PREFIX, PREFIX + NEW - CH):
        pairs = CH * base + CH * (CH + 1) // 2
        flops = pairs * N_Q * 4 * HD
        t_ref = timeit(lambda it: ref.q27ref_attn_prefill_T(
            qT.data_ptr(), Q_STRIDE, N_Q * Q_STRIDE, ktab.data_ptr(), vtab.data_ptr(), outT.data_ptr(),
            N_Q * HD, part.data_ptr(), base, 0, CH, N_Q, N_KV, HD, SCALE, st, KV_F16), max(2, args.steps // 5))
        t_ours = timeit(lambda it: Q.attn_prefill_T(qT, Q_STRIDE, N_Q * Q_STRIDE, ktab, vtab, outT, N_Q * HD,
                                                    part, base, 0, CH, N_Q, N_KV, HD, SCALE, kvk=KV_F16),
                        max(2, args.steps // 5))
        out["workloads"][f"c4 chunk at base {base}"] = {
            "reference_ms": round(t_ref, 4), "ours_ms": round(t_ours, 4), "speedup": round(t_ref / t_ours, 2),
            "reference_TFLOPs": round(flops / t_ref / 1e9, 1), "ours_TFLOPs": round(flops / t_ours / 1e9, 1)}
    print(json.dumps(out), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=30)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--repeats", type=int, default=50,
                    help="timed regions of --steps steps each; the median region is reported")
    ap.add_argument("--workload", default=None, choices=sorted(DECODE) + ["c4"],
                    help="measure this workload alone (default: c3 as the line, the others under `configs`)")
    ap.add_argument("--impl", default="ours", choices=["ours", "reference", "reference-gpu"])
    ap.add_argument("--no-cpu", action="store_true", help="skip the oracle checks and the cpu_baseline leg")
    ap.add_argument("--no-graph", action="store_true",
                    help="launch every step directly instead of replaying CUDA graphs")
    ap.add_argument("--exchange", default="peer", choices=["peer", "nccl"],
                    help="N > 1: how the ranks' partials meet (peer-memory mailboxes or NCCL)")
    args = ap.parse_args()
    if args.warmup < 3 and args.impl == "ours":
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    elif args.impl == "reference-gpu":
        run_reference_gpu(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
