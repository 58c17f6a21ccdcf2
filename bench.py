#!/usr/bin/env python
"""Headline benchmark: BASELINE config 3, the int4 paged decode step at batch 256 x 4k context.

Workload (per GPU; requests are partitioned across GPUs, so N GPUs serve N x 256 sequences -- weak scaling):
Llama-3.1-8B attention geometry (32 q heads, 8 kv heads, head_dim 128), 32 layers, int4 records with 16-token
pages, 256 sequences of 4096 cached tokens each, a seeded random block table.  K/V/q are bf16 N(0, 1); keys carry
per-channel offsets N(0, 2) plus 2 outlier channels at +-15 per kv head (synthetic data of the config's shape --
there is no dataset in this benchmark).  One step = for each of the 32 layers: quantize-on-write of one new token
per sequence (append) and fused dequant decode attention over the whole cache.  The step is captured once in a CUDA
graph and replayed; the 44 GB of records per step are far larger than L2, so no flush is needed between steps.

Printed (rank 0, one JSON line): value = packed-KV GB/s of the whole job (all ranks' record bytes / max-over-ranks
device time), us per layer-step, decode tokens/s; e2e = the same metric through the public API with per-step host
inputs (pinned) copied in and outputs copied back inside the timed region (each step's copies on a copy stream,
overlapped with the neighbouring steps' kernels as a serving loop runs them); roofline of the decode kernel (achieved
algorithmic bytes / its CUDA-event duration vs the measured HBM copy peak); the CPU oracle timed on a bounded sample
(cpu_baseline); clocks sampled with nvidia-smi during the timed region.

    python bench.py [--gpus N] [--steps K] [--warmup W]
    python bench.py --workload long           # BASELINE config 4 (kv heads partitioned over the GPUs)
    python bench.py --workload mix            # BASELINE config 5 (serving mix: prompt writes + ragged decode)
    python bench.py --workload c1 | c2        # BASELINE configs 1 and 2 (single-layer Qwen2.5-7B geometry)
    python bench.py --workload unpack         # prefill with history: records -> packed bf16 K/V (unpack)
    python bench.py --impl reference          # the reference's CPU algorithm (C restatement) on the host cores
    torchrun --nproc-per-node N bench.py --gpus N ...
"""
from __future__ import annotations

import argparse
import datetime
import json
import math
import os
import subprocess
import sys
import time
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "int4 decode attn: packed-KV HBM GB/s (% of 8 TB/s) and µs/layer-step; tokens/s 1–8 GPU"
NOMINAL_HBM_GBS = 8000.0
FALLBACK_HBM_GBS = 6650.0
# split-KV decodes merge their splits with a separate combine launch (as the reference's kush_combine);
# --combine fused merges them inside the decode launch (Ops.decode(fused=True)), measured slower on B200
FUSED_COMBINE = False


# ---------------------------------------------------------------- workload
class Geometry:
    def __init__(self, a, hkv: int = 8):
        self.L, self.B, self.N, self.P = a.layers, a.batch, a.context, a.page
        self.HQ, self.HKV, self.D, self.bits = 4 * hkv, hkv, 128, 4
        self.G = self.HQ // self.HKV
        self.DC = self.D // 2 if self.bits == 4 else self.D
        self.RB = 2 * self.P * self.DC + 4 * self.D + 4 * self.P
        self.long = getattr(a, "workload", "batch") == "long"

    def packed_bytes(self, n: int, seqs: int | None = None) -> int:
        """Packed-KV bytes one decode reads for `seqs` sequences of n tokens: full pages' records plus the partial
        page's exact-K tail rows, V codes and V scale/bias (per kv head)."""
        seqs = self.B if seqs is None else seqs
        full, r = divmod(n, self.P)
        return seqs * self.HKV * (full * self.RB + r * (2 * self.D + self.DC + 4))

    def decode_algorithmic_bytes(self, n: int) -> int:
        """Bytes per decode launch: packed KV + q in + out (bf16)."""
        return self.packed_bytes(n) + self.B * self.HQ * self.D * 2 * 2

    def describe(self) -> dict:
        if self.long:
            return {"workload": f"BASELINE config 4: Qwen3-8B attention geometry, {self.L} layers, int4, batch {self.B} x "
                                f"{self.N} context, page {self.P}; kv heads partitioned over the GPUs, one step = append "
                                "+ split-KV decode + output all_gather per layer",
                    "model": "Qwen3-8B (attention geometry only: 32 q heads, 8 kv heads, head_dim 128)",
                    "seq_len": self.N, "global_batch": self.B, "layers": self.L, "page": self.P, "bits": self.bits,
                    "kv_heads_per_gpu": self.HKV, "head_dim": self.D,
                    "l2": "inputs larger than L2 (records of all layers per step, no flush needed)"}
        return {"workload": f"BASELINE config 3: Llama-3.1-8B attention geometry, {self.L} layers, int4, "
                            f"batch {self.B} x {self.N} context, page {self.P}; one step = append + decode per layer",
                "model": "Llama-3.1-8B (attention geometry only: 32 q heads, 8 kv heads, head_dim 128)",
                "global_batch": None, "seq_len": self.N, "batch_per_gpu": self.B, "layers": self.L,
                "page": self.P, "bits": self.bits, "q_heads": self.HQ, "kv_heads": self.HKV, "head_dim": self.D,
                "l2": "inputs larger than L2 (records of 32 layers per step, no flush needed)"}


def batch_config(geo: Geometry, world: int, rotate: str = "none") -> dict:
    """The `config` of a config-3 JSON line; both arms print this same dict (the reference arm describes its
    bounded host sample in its cpu_baseline)."""
    return {**geo.describe(), "global_batch": geo.B * world,
            "parallelism": f"requests partitioned over {world} GPU(s), no collective in the step",
            "rotation": {"none": "off (as BASELINE)", "fused": "Walsh-Hadamard inside the append and decode kernels",
                         "unfused": "Walsh-Hadamard by fwht launches around append and decode"}[rotate]}


def key_offsets(geo: Geometry, gen: torch.Generator, device) -> torch.Tensor:
    """Per-channel key offsets N(0, 2) plus 2 outlier channels at +-15 per kv head ([Hkv, D])."""
    off = torch.randn(geo.HKV, geo.D, generator=gen) * 2
    for h in range(geo.HKV):
        idx = torch.randperm(geo.D, generator=gen)[:2]
        off[h, idx] = 15 * torch.sign(torch.randn(2, generator=gen))
    return off.to(device)


class Engine:
    """32 layers of cache state on one GPU, filled with the context, plus the per-step inputs."""

    def __init__(self, geo: Geometry, device: torch.device, seed: int, extra_tokens: int, rotate: str = "none"):
        from kushkash_b200 import Ops
        self.geo, self.dev, self.rotate = geo, device, rotate
        g = geo
        self.ops = Ops(device, g.D, g.bits, g.G, torch.bfloat16, g.P)
        gen = torch.Generator().manual_seed(seed)
        # room for every token the run appends (warm-up, timed and e2e steps), so no position leaves the table
        self.pages_per_seq = -(-(g.N + extra_tokens) // g.P)
        n_blocks = g.B * self.pages_per_seq
        perm = torch.randperm(n_blocks, generator=gen).to(torch.int32)
        self.block_table = perm.view(g.B, self.pages_per_seq).to(device)
        self.tail_idx = torch.arange(g.B, dtype=torch.int32, device=device)
        self.pool = torch.zeros(g.L, n_blocks, g.HKV, g.RB, dtype=torch.uint8, device=device)
        self.tail_k = torch.zeros(g.L, g.B, g.HKV, g.P, g.D, dtype=torch.bfloat16, device=device)
        self.seq_lens = torch.zeros(g.L, g.B, dtype=torch.int32, device=device)
        self.offsets = key_offsets(g, gen, device)
        self.scale = 1.0 / math.sqrt(g.D)
        self.ns = self.ops.splits(g.B, g.HKV, g.N // g.P)
        self.fused = FUSED_COMBINE
        # zeros: the fused combine's counters at the end of the work buffer start at 0
        self.work = torch.zeros(max(1, self.ops.work_size(g.B, g.HKV, self.ns, self.fused)), device=device)
        dgen = torch.Generator(device=device).manual_seed(seed + 1)
        self._fill(dgen)
        # per-step inputs: new token K/V rows and q per layer (bf16), outputs
        self.k_new = self._keys(torch.randn(g.L, g.B, g.HKV, g.D, generator=dgen, device=device)).to(torch.bfloat16)
        self.v_new = torch.randn(g.L, g.B, g.HKV, g.D, generator=dgen, device=device).to(torch.bfloat16)
        self.q = torch.randn(g.L, g.B, g.HQ, g.D, generator=dgen, device=device).to(torch.bfloat16)
        self.out = torch.empty_like(self.q)
        self.set_rotation(rotate)

    def _keys(self, x: torch.Tensor) -> torch.Tensor:
        return x + self.offsets.to(x.dtype)

    def _fill(self, dgen) -> None:
        """Bulk quantize-on-write of the first N tokens of every layer (chunks of 1024 tokens)."""
        g = self.geo
        chunk = 1024
        for layer in range(g.L):
            n = 0
            while n < g.N:
                T = min(chunk, g.N - n)
                k = self._keys(torch.randn(g.B, T, g.HKV, g.D, generator=dgen, device=self.dev)).to(torch.bfloat16)
                v = torch.randn(g.B, T, g.HKV, g.D, generator=dgen, device=self.dev).to(torch.bfloat16)
                if self.rotate != "none":       # a rotated cache holds K H and V H
                    k, v = self.ops.fwht(k, out=k), self.ops.fwht(v, out=v)
                self.seq_lens[layer].fill_(n + T)
                pages = torch.arange(n // g.P, (n + T - 1) // g.P + 1, dtype=torch.int32, device=self.dev)
                job_seq = torch.arange(g.B, dtype=torch.int32, device=self.dev).repeat_interleave(pages.numel())
                qsl = torch.arange(g.B + 1, dtype=torch.int32, device=self.dev) * T
                self.ops.write(k.view(g.B * T, g.HKV, g.D), v.view(g.B * T, g.HKV, g.D), qsl, self.seq_lens[layer],
                               self.tail_idx, job_seq, pages.repeat(g.B), self.pool[layer], self.block_table,
                               self.tail_k[layer])
                n += T
        torch.cuda.synchronize(self.dev)

    rotate = "none"         # "fused": rotation inside the append / decode kernels; "unfused": fwht launches around

    def step(self) -> None:
        """One decode step: per layer, append one token per sequence, then decode attention (2 launches/layer)."""
        g, ops = self.geo, self.ops
        for layer in range(g.L):
            k, v = self.k_new[layer], self.v_new[layer]
            if self.rotate == "unfused":
                k, v = ops.fwht(k, out=self.rk), ops.fwht(v, out=self.rv)
            ops.append(k, v, self.seq_lens[layer], self.tail_idx, self.pool[layer], self.block_table,
                       self.tail_k[layer], pos_offset=0, advance=True, rotate=self.rotate == "fused")
            self._decode(layer)

    def appends_only(self) -> None:
        """The appends of one step (and their rotations), writing the same rows without advancing the lengths: the
        part of a step that is not the decode, for the decode's share of the timed region."""
        g, ops = self.geo, self.ops
        for layer in range(g.L):
            k, v = self.k_new[layer], self.v_new[layer]
            if self.rotate == "unfused":
                k, v = ops.fwht(k, out=self.rk), ops.fwht(v, out=self.rv)
            ops.append(k, v, self.seq_lens[layer], self.tail_idx, self.pool[layer], self.block_table,
                       self.tail_k[layer], pos_offset=0, advance=False, rotate=self.rotate == "fused")

    def _decode(self, layer: int) -> None:
        g, ops = self.geo, self.ops
        q = ops.fwht(self.q[layer], out=self.rq) if self.rotate == "unfused" else self.q[layer]
        ops.decode(q, self.out[layer], self.pool[layer], self.block_table, self.seq_lens[layer], self.tail_idx,
                   self.tail_k[layer], self.scale, self.ns, self.work, rotate=self.rotate == "fused", fused=self.fused)
        if self.rotate == "unfused":
            ops.fwht(self.out[layer], out=self.out[layer])

    def set_rotation(self, mode: str) -> None:
        self.rotate = mode
        if mode == "unfused":                   # scratch rows for the rotated k, v, q of a layer
            self.rk, self.rv = torch.empty_like(self.k_new[0]), torch.empty_like(self.v_new[0])
            self.rq = torch.empty_like(self.q[0])

    def decode_only(self) -> None:
        """The decode launches alone (with rotation fused into them when it is on), for the kernel's roofline."""
        g, ops = self.geo, self.ops
        for layer in range(g.L):
            ops.decode(self.q[layer], self.out[layer], self.pool[layer], self.block_table, self.seq_lens[layer],
                       self.tail_idx, self.tail_k[layer], self.scale, self.ns, self.work, rotate=self.rotate == "fused",
                       fused=self.fused)

    def launches_per_step(self) -> int:
        combine = 1 if self.ns > 1 and not self.fused else 0
        return self.geo.L * (2 + combine + (4 if self.rotate == "unfused" else 0))


class OverlappedIO:
    """Per-step host inputs and outputs of an e2e figure, overlapped with the device work the way a serving loop runs:
    step i+1's inputs cross PCIe on a copy stream (pinned host -> device staging) while step i computes, and step i's
    outputs return (device staging -> pinned host) while step i+1 computes.  Each step copies its inputs from the
    staging into the buffers its (captured) kernels read, and its outputs into the output staging, on the compute
    stream.  Every byte still crosses PCIe inside the timed region: the loop ends with the compute stream waiting for
    the copy stream."""

    def __init__(self, inputs: dict[str, torch.Tensor], output, device: torch.device):
        self.inputs, self.device = inputs, device
        self.outputs = list(output) if isinstance(output, (list, tuple)) else [output]
        self.host_in = {k: v.cpu().pin_memory() for k, v in inputs.items()}
        self.stage_in = {k: torch.empty_like(v) for k, v in inputs.items()}
        self.stage_out = [torch.empty_like(o) for o in self.outputs]
        self.host_out = [torch.empty(o.shape, dtype=o.dtype).pin_memory() for o in self.outputs]
        self.copy_stream = torch.cuda.Stream(device)
        self.h2d_bytes = sum(t.numel() * t.element_size() for t in self.host_in.values())
        self.d2h_bytes = sum(t.numel() * t.element_size() for t in self.host_out)

    def _prefetch(self, main) -> torch.cuda.Event:
        self.copy_stream.wait_stream(main)                  # the staging has been consumed
        with torch.cuda.stream(self.copy_stream):
            for k, t in self.host_in.items():
                self.stage_in[k].copy_(t, non_blocking=True)
        return self.copy_stream.record_event()

    def run(self, steps: int, compute) -> None:
        main = torch.cuda.current_stream(self.device)
        in_ready, out_done = self._prefetch(main), None
        for i in range(steps):
            main.wait_event(in_ready)
            for k, t in self.inputs.items():
                t.copy_(self.stage_in[k])
            if i + 1 < steps:
                in_ready = self._prefetch(main)
            outs = compute()                                # a step may name this step's output buffers
            if out_done is not None:
                main.wait_event(out_done)                   # the previous outputs have left the staging
            for s, o in zip(self.stage_out, self.outputs if outs is None else outs):
                s.copy_(o)
            self.copy_stream.wait_stream(main)
            with torch.cuda.stream(self.copy_stream):
                for h, s in zip(self.host_out, self.stage_out):
                    h.copy_(s, non_blocking=True)
            out_done = self.copy_stream.record_event()
        main.wait_stream(self.copy_stream)


class PingPongIO:
    """Per-step host inputs and outputs of an e2e figure with two sets of the step's input and output buffers, each
    read and written by its own captured graph: step i runs graph i % 2, while step i+1's inputs cross PCIe straight
    into the other set (pinned host -> device, one copy stream) and step i-1's outputs leave the other set (device ->
    pinned host, a second copy stream, so both directions of PCIe are busy at once).  No staging copies on the
    device.  A set's inputs are overwritten only after the graph that read them finished, and its outputs only after
    they were copied out.  Every byte still crosses PCIe inside the timed region: the loop ends with the compute
    stream waiting for both copy streams."""

    def __init__(self, sets: list[dict[str, torch.Tensor]], outs: list[torch.Tensor], graphs: list, device):
        self.sets, self.outs, self.graphs, self.device = sets, outs, graphs, device
        self.host_in = {k: v.cpu().pin_memory() for k, v in sets[0].items()}
        self.host_out = torch.empty(outs[0].shape, dtype=outs[0].dtype).pin_memory()
        self.h2d_stream, self.d2h_stream = torch.cuda.Stream(device), torch.cuda.Stream(device)
        self.h2d_bytes = sum(t.numel() * t.element_size() for t in self.host_in.values())
        self.d2h_bytes = self.host_out.numel() * self.host_out.element_size()

    def _h2d(self, p: int, after) -> torch.cuda.Event:
        if after is not None:
            self.h2d_stream.wait_event(after)                 # the graph that last read set p has finished
        with torch.cuda.stream(self.h2d_stream):
            for k, t in self.host_in.items():
                self.sets[p][k].copy_(t, non_blocking=True)
        return self.h2d_stream.record_event()

    def run(self, steps: int) -> None:
        main = torch.cuda.current_stream(self.device)
        done = [main.record_event(), main.record_event()]    # graph of set p finished
        out_free = [None, None]                              # outputs of set p copied out
        ready = [self._h2d(0, done[0]), None]
        for i in range(steps):
            p = i % 2
            if i + 1 < steps:
                ready[1 - p] = self._h2d(1 - p, done[1 - p])
            main.wait_event(ready[p])
            if out_free[p] is not None:
                main.wait_event(out_free[p])
            self.graphs[p].replay()
            done[p] = main.record_event()
            self.d2h_stream.wait_event(done[p])
            with torch.cuda.stream(self.d2h_stream):
                self.host_out.copy_(self.outs[p], non_blocking=True)
            out_free[p] = self.d2h_stream.record_event()
        main.wait_stream(self.h2d_stream)
        main.wait_stream(self.d2h_stream)


class CapturedIO:
    """Per-step host inputs and outputs of an e2e figure for steps too short to overlap from the host: the copies from
    pinned host memory and back are captured into the step's CUDA graph around its kernels, so one replay does
    host -> device, the step, device -> host (serially, with no host work per step)."""

    def __init__(self, inputs: dict[str, torch.Tensor], output: torch.Tensor, device: torch.device, step):
        self.host_in = {k: v.cpu().pin_memory() for k, v in inputs.items()}
        self.host_out = torch.empty(output.shape, dtype=output.dtype).pin_memory()
        self.h2d_bytes = sum(t.numel() * t.element_size() for t in self.host_in.values())
        self.d2h_bytes = self.host_out.numel() * self.host_out.element_size()

        def body():
            for k, t in self.host_in.items():
                inputs[k].copy_(t, non_blocking=True)
            step()
            self.host_out.copy_(output, non_blocking=True)
        self.graph = capture(body, device)

    def run(self, steps: int, _compute=None) -> None:
        for _ in range(steps):
            self.graph.replay()


def capture(fn, device) -> torch.cuda.CUDAGraph:
    """Capture fn's launches (the kernels launch on torch's current stream, the capture stream) without running them."""
    torch.cuda.synchronize(device)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        fn()
    return g


# ---------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi samples (every 200 ms) of this GPU's SM clock and throttle reasons during the timed region."""
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.proc = None
        self.idx = self._smi_index(device)
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "200"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None

    @staticmethod
    def _smi_index(device: int) -> str | None:
        try:
            bus = torch.cuda.get_device_properties(device).pci_bus_id
            dom = torch.cuda.get_device_properties(device).pci_domain_id
            dev = torch.cuda.get_device_properties(device).pci_device_id
            want = f"{dom:08x}:{bus:02x}:{dev:02x}".upper()
            r = subprocess.run(["nvidia-smi", "--query-gpu=index,pci.bus_id", "--format=csv,noheader"],
                               capture_output=True, text=True, timeout=20)
            for line in r.stdout.strip().splitlines():
                i, b = (x.strip() for x in line.split(","))
                if b.upper().startswith(want):
                    return i
        except Exception:
            pass
        return None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.3)
        self.proc.terminate()
        try:
            out, _ = self.proc.communicate(timeout=10)
        except subprocess.TimeoutExpired:
            self.proc.kill()
            out, _ = self.proc.communicate()
        rows = [[x.strip() for x in ln.split(",")] for ln in out.strip().splitlines() if ln.count(",") >= 8]
        if self.idx is not None:
            rows = [r for r in rows if r[0] == self.idx] or rows
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        sm, mx, reasons = [], None, set()
        for r in rows:
            try:
                sm.append(float(r[1]))
                mx = float(r[2])
            except ValueError:
                continue
            for name, val in zip(names, r[5:9]):
                if val.lower().startswith("active"):
                    reasons.add(name)
        sm.sort()
        return {"sm_mhz": sm[len(sm) // 2] if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


# ---------------------------------------------------------------- CPU baseline (the oracle, on a bounded sample)
def cpu_sample_from_engine(eng: Engine, seqs: int):
    """Layer 0 of the first `seqs` sequences, copied to the host in the oracle's fp32 layout."""
    g = eng.geo
    n = int(eng.seq_lens[0, 0].item())
    pages = -(-n // g.P)
    blk = eng.block_table[:seqs, :pages].long()
    pool = eng.pool[0][blk.reshape(-1)].cpu().contiguous()                       # [seqs*pages, H, RB]
    bt = torch.arange(seqs * pages, dtype=torch.int32).view(seqs, pages)
    tail = eng.tail_k[0, :seqs].float().cpu().contiguous()
    q = eng.q[0, :seqs].float().cpu().contiguous()
    sl = torch.full((seqs,), n, dtype=torch.int32)
    return dict(pool=pool, bt=bt, tail=tail, q=q, seq_lens=sl, tail_idx=torch.arange(seqs, dtype=torch.int32), n=n)


def cpu_sample_synthetic(geo: Geometry, seqs: int, seed: int, extra_tokens: int):
    """The same workload built on the host by the oracle itself (bulk write of N tokens for `seqs` sequences)."""
    from oracle.kush_oracle import OracleOps
    g = geo
    gen = torch.Generator().manual_seed(seed)
    off = key_offsets(g, gen, "cpu")
    ops = OracleOps(g.D, g.bits, g.G, g.P)
    pages = -(-(g.N + extra_tokens) // g.P)
    pool = torch.zeros(seqs * pages, g.HKV, g.RB, dtype=torch.uint8)
    bt = torch.randperm(seqs * pages, generator=gen).to(torch.int32).view(seqs, pages)
    tail = torch.zeros(seqs, g.HKV, g.P, g.D)
    ti = torch.arange(seqs, dtype=torch.int32)
    sl = torch.zeros(seqs, dtype=torch.int32)
    k = (torch.randn(seqs, g.N, g.HKV, g.D, generator=gen) + off).bfloat16().float()
    v = torch.randn(seqs, g.N, g.HKV, g.D, generator=gen).bfloat16().float()
    sl.fill_(g.N)
    pg = torch.arange(0, (g.N - 1) // g.P + 1, dtype=torch.int32)
    ops.write(k.view(-1, g.HKV, g.D), v.view(-1, g.HKV, g.D), torch.arange(seqs + 1, dtype=torch.int32) * g.N, sl, ti,
              torch.arange(seqs, dtype=torch.int32).repeat_interleave(pg.numel()), pg.repeat(seqs), pool, bt, tail)
    q = torch.randn(seqs, g.HQ, g.D, generator=gen).bfloat16().float()
    return dict(pool=pool, bt=bt, tail=tail, q=q, seq_lens=sl, tail_idx=ti, n=g.N,
                k_new=(torch.randn(seqs, g.HKV, g.D, generator=gen) + off).bfloat16().float(),
                v_new=torch.randn(seqs, g.HKV, g.D, generator=gen).bfloat16().float())


def time_cpu_decode(geo: Geometry, smp: dict, budget_s: float, with_append: bool = False) -> dict:
    """Oracle decode (one task per (sequence, kv head) over all host threads) repeated for ~budget_s seconds."""
    from oracle.kush_oracle import OracleOps, set_threads
    g = geo
    cores = set_threads(host_threads())
    ops = OracleOps(g.D, g.bits, g.G, g.P)
    seqs = smp["q"].shape[0]
    out = torch.empty_like(smp["q"])
    iters, t0, byts = 0, time.perf_counter(), 0
    while True:
        if with_append:
            ops.append(smp["k_new"], smp["v_new"], smp["seq_lens"], smp["tail_idx"], smp["pool"], smp["bt"],
                       smp["tail"], pos_offset=0, advance=True)
        ops.decode(smp["q"], out, smp["pool"], smp["bt"], smp["seq_lens"], smp["tail_idx"], smp["tail"],
                   1.0 / math.sqrt(g.D))
        byts += g.packed_bytes(int(smp["seq_lens"][0]), seqs)
        iters += 1
        el = time.perf_counter() - t0
        if el >= budget_s or iters >= 10000:
            break
    return {"value": byts / el / 1e9, "unit": "GB/s", "cores": cores, "kind": "port",
            "sample": f"layer-steps of {seqs} of the {g.B} sequences x {g.HKV} kv heads at {smp['n']} tokens "
                      f"({iters} decode calls{' + appends' if with_append else ''}, {el:.1f} s)",
            "seconds_per_call": el / iters}


def host_threads() -> int:
    """Host cores this process may run on.  Passed to the oracle explicitly: torchrun sets OMP_NUM_THREADS=1 for its
    ranks, which would otherwise leave a CPU baseline timed under torchrun on one core."""
    try:
        return max(1, len(os.sched_getaffinity(0)))
    except AttributeError:
        return max(1, os.cpu_count() or 1)


# ---------------------------------------------------------------- measured peaks
def hbm_peak() -> tuple[float, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    try:
        return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def ncu_traffic() -> float | None:
    """DRAM bytes per decode launch at this workload from the committed ncu summary (profiles/), if present."""
    p = ROOT / "profiles" / "decode_config3_traffic.json"
    try:
        return float(json.loads(p.read_text())["bytes_per_launch_config3"])
    except Exception:
        return None


# ---------------------------------------------------------------- main
def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--batch", type=int, default=256, help="sequences per GPU (config 3: 256)")
    ap.add_argument("--context", type=int, default=4096, help="cached tokens per sequence (config 3: 4096)")
    ap.add_argument("--layers", type=int, default=32, help="layers per step (config 3: 32)")
    ap.add_argument("--page", type=int, default=16, help="tokens per page (config 3: 16)")
    ap.add_argument("--cpu-seconds", type=float, default=12.0, help="CPU-baseline sample budget")
    ap.add_argument("--cpu-seqs", type=int, default=32, help="sequences in the CPU-baseline sample")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--launch-order", choices=["longest", "natural"], default="longest",
                    help="ragged workloads (configs 2, 5): decode CTAs take the sequences longest first (an order "
                         "computed once per step) or in their natural order")
    ap.add_argument("--rotate", choices=["none", "fused", "unfused"], default="none",
                    help="config 3 with the Walsh-Hadamard rotation of kushkash's 4-bit default: inside the append and "
                         "decode kernels (fused) or as fwht launches around them (unfused); BASELINE runs without")
    ap.add_argument("--gather", choices=["peer", "nccl"], default="peer",
                    help="config 4 on N > 1 GPUs: outputs gathered by the combine's stores into every rank's buffer "
                         "over NVLink (one CUDA graph per step) or by an NCCL all_gather per layer (eager steps)")
    ap.add_argument("--combine", choices=["fused", "launch"], default="launch",
                    help="split-KV decodes: the splits merged by a separate combine launch, as the reference does "
                         "(launch), or by the last CTA of each unit inside the decode launch (fused)")
    ap.add_argument("--workload", choices=["batch", "long", "mix", "c1", "c2", "unpack"], default="batch",
                    help="batch: config 3 (default, requests partitioned); long: config 4 (kv heads partitioned); "
                         "mix: config 5 (serving mix); c1, c2: configs 1 and 2 (single layer; requests partitioned); "
                         "unpack: prefill with history (packed K/V for a prefill attention)")
    a = ap.parse_args()
    global FUSED_COMBINE
    FUSED_COMBINE = a.combine == "fused"
    if a.workload == "long":
        for k, v in (("batch", 4), ("context", 131072), ("page", 32), ("layers", 8)):
            if getattr(a, k) == ap.get_default(k):
                setattr(a, k, v)
    if a.workload == "mix" and a.layers == ap.get_default("layers"):
        a.layers = 4
    if a.workload == "unpack" and a.layers == ap.get_default("layers"):
        a.layers = 8
    if a.warmup < 3 and a.impl == "ours":
        print("bench.py: --warmup < 3 is raised to 3 (timing rule)", file=sys.stderr)
        a.warmup = 3
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    geo = Geometry(a)

    if a.impl == "reference":
        if a.workload == "unpack":
            run_reference_unpack(a, world, rank)
        else:
            run_reference(a, geo, world, rank)
        return
    if a.workload == "unpack":
        run_unpack(a, world, rank, local)
        return
    if a.workload == "long":
        run_long(a, world, rank, local)
        return
    if a.workload in ("mix", "c1", "c2"):
        if a.workload == "c2" and a.steps == ap.get_default("steps"):
            a.steps = 16                           # config 2: 16 consecutive steps timed
        run_ragged(a, world, rank, local, a.workload)
        return

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist = None
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=120))
    eng = Engine(geo, dev, seed=1234 + rank, extra_tokens=a.warmup + 2 * a.steps + 8, rotate=a.rotate)

    # warm-up (eager, then capture the step)
    for _ in range(a.warmup - 1):
        eng.step()
    graph = capture(eng.step, dev)              # capture runs no kernels; replays below each do one step
    n0 = int(eng.seq_lens[0, 0].item())

    def barrier():
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize(dev)

    # ---- timed region: K graph replays of the full step
    sampler = ClockSampler(local)               # started before the barrier: its spawn cannot skew the ranks
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(a.steps):
        graph.replay()
    e1.record()
    torch.cuda.synchronize(dev)
    clocks = sampler.stop()
    barrier()
    ms = e0.elapsed_time(e1)
    bytes_local = sum(geo.packed_bytes(n0 + i + 1) for i in range(a.steps)) * geo.L
    # ---- decode-kernel roofline: the decode's time in the timed region -- the timed steps less their appends (one
    # step's appends timed right after as a graph, CUDA events on the launching stream) -- per decode launch.  The
    # gaps between launches are counted as decode time.  The decode bytes are those of the middle timed step.
    agraph = capture(eng.appends_only, dev)
    agraph.replay()
    torch.cuda.synchronize(dev)
    a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a0.record()
    for _ in range(3):
        agraph.replay()
    a1.record()
    torch.cuda.synchronize(dev)
    app_ms = a0.elapsed_time(a1) / 3
    dec_ms = (ms / a.steps - app_ms) / geo.L
    dec_bytes = geo.decode_algorithmic_bytes(n0 + (a.steps + 1) // 2)
    del agraph
    # and, for comparison, the decodes alone back to back (a graph of the 32 launches after the timed region, at the
    # clocks the board's power limit leaves after the seconds of load before it)
    dgraph = capture(eng.decode_only, dev)
    dgraph.replay()
    torch.cuda.synchronize(dev)
    reps = max(2, a.steps)
    d0, d1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    d0.record()
    for _ in range(reps):
        dgraph.replay()
    d1.record()
    torch.cuda.synchronize(dev)
    dec_only_ms = d0.elapsed_time(d1) / (reps * geo.L)
    # ---- e2e: public API from pinned host buffers, every step's copies inside the timed region, overlapped with the
    # neighbouring steps' kernels: two sets of inputs / outputs, one captured step graph per set (PingPongIO)
    names = ("q", "k_new", "v_new", "out")
    set0 = {k: getattr(eng, k) for k in names}
    set1 = {k: torch.empty_like(v) for k, v in set0.items()}
    for k, v in set1.items():
        if k != "out":
            v.copy_(set0[k])
    graphs = [graph]
    for k in names:
        setattr(eng, k, set1[k])
    graphs.append(capture(eng.step, dev))
    for k in names:
        setattr(eng, k, set0[k])
    io = PingPongIO([{k: st[k] for k in names[:3]} for st in (set0, set1)], [set0["out"], set1["out"]], graphs, dev)
    io.run(2)
    barrier()
    n_e2e = int(eng.seq_lens[0, 0].item())
    x0, x1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    x0.record()
    io.run(a.steps)
    x1.record()
    torch.cuda.synchronize(dev)
    barrier()
    e2e_ms = x0.elapsed_time(x1)
    e2e_bytes_local = sum(geo.packed_bytes(n_e2e + i + 1) for i in range(a.steps)) * geo.L
    h2d, d2h = io.h2d_bytes, io.d2h_bytes

    if dist is not None:
        t = torch.tensor([ms, e2e_ms, dec_ms, dec_only_ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, e2e_ms, dec_ms, dec_only_ms = (float(x) for x in t.tolist())
        b = torch.tensor([bytes_local, e2e_bytes_local], device=dev, dtype=torch.float64)
        dist.all_reduce(b)
        bytes_all, e2e_bytes_all = (float(x) for x in b.tolist())
    else:
        bytes_all, e2e_bytes_all = float(bytes_local), float(e2e_bytes_local)

    cpu = None
    if rank == 0 and world == 1 and not a.no_cpu_baseline:
        smp = cpu_sample_from_engine(eng, min(a.cpu_seqs, geo.B))
        cpu = time_cpu_decode(geo, smp, a.cpu_seconds)
        cpu.pop("seconds_per_call", None)

    if rank == 0:
        peak, peak_kind = hbm_peak()
        value = bytes_all / (ms / 1e3) / 1e9
        ms_step = ms / a.steps
        achieved = dec_bytes / (dec_ms / 1e3) / 1e9
        traffic = ncu_traffic()
        line = {
            "metric": METRIC, "value": round(value, 1), "unit": "GB/s", "n_gpus": world, "steps": a.steps,
            "warmup": a.warmup, "ms_per_step": round(ms_step, 4), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "int4 records, bf16 q/k/v, fp32 softmax",
            "data": "synthetic (seeded bf16 N(0,1) K/V/q with per-channel key offsets, BASELINE config 3 shapes)",
            "config": batch_config(geo, world, a.rotate),
            "pct_of_8TBs": round(100 * value / world / NOMINAL_HBM_GBS, 1),
            "us_per_layer_step": round(ms_step * 1e3 / geo.L, 2),
            "decode_tokens_per_s": round(geo.B * world / (ms_step / 1e3), 1),
            "e2e": {"value": round(e2e_bytes_all / (e2e_ms / 1e3) / 1e9, 1), "unit": "GB/s",
                    "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "ms_per_step": round(e2e_ms / a.steps, 4)},
            "roofline": {"kernel": "kush_sm100_decode", "bound": "hbm", "achieved": round(achieved, 1),
                         "peak": peak, "peak_kind": f"{peak_kind} (HBM copy, MEASURED_PEAKS.json)" if peak_kind ==
                         "measured" else "fallback", "unit": "GB/s", "frac": round(achieved / peak, 4),
                         "traffic": traffic, "algorithmic_bytes_per_launch": dec_bytes,
                         "us_per_launch": round(dec_ms * 1e3, 2),
                         "timing": "timed steps less one step's appends (graph, events), per decode launch",
                         "us_appends_per_step": round(app_ms * 1e3, 2),
                         "us_per_launch_decodes_back_to_back": round(dec_only_ms * 1e3, 2)},
            "cpu_baseline": cpu,
            "clocks": clocks,
            "gpu_launches": a.steps * eng.launches_per_step(),
            "decode_kernel": "tensor cores" if eng.ops.cfg.tensor_cores else "cuda cores",
            "n_splits": eng.ns, "split_combine": "fused" if eng.fused else "launch",
        }
        print(json.dumps(line), flush=True)
    del graph, dgraph, graphs, io
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


def run_long(a, world: int, rank: int, local: int) -> None:
    """4 sequences of 131072 tokens; rank r owns kv heads [8r/N, 8(r+1)/N) of every sequence and
    layer, runs append + split-KV decode for them, and the per-layer [4, 32/N, 128] outputs are all_gathered over NCCL
    (the only collective).  Strong scaling: the total work is fixed as N grows."""
    from kushkash_b200.shard import PeerGather, decode_gathered, gather_heads, kv_head_range
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist = None
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=120))
    h0, h1 = kv_head_range(8, rank, world)
    geo = Geometry(a, hkv=h1 - h0)
    full = Geometry(a, hkv=8)
    eng = Engine(geo, dev, seed=4321 + rank, extra_tokens=a.warmup + 2 * a.steps + 8)
    pg = None
    if dist is not None and a.gather == "peer":                 # gathered by the combine's peer stores
        eng.fused = False                                       # the gather is the combine
        if eng.ns < 2:
            eng.ns = 2
            eng.work = torch.empty(eng.ops.work_size(geo.B, geo.HKV, 2), device=dev)
        # two sets of per-layer slots, alternating per step: a peer's stores of step k+1 land in the other set, and
        # it cannot start step k+2 before this rank has run step k+1's combines, which its stream orders after the
        # reads of step k's outputs (PeerGather's slot-reuse rule)
        pg = PeerGather(geo.B, full.HQ, geo.D, torch.bfloat16, slots=2 * geo.L)
        out_sets = [pg.outs[:geo.L], pg.outs[geo.L:]]
    else:
        outs = [torch.empty(geo.B, full.HQ, geo.D, dtype=torch.bfloat16, device=dev) for _ in range(geo.L)]
        out_sets = [outs, outs]

    def step(parity: int = 0):
        for layer in range(geo.L):
            eng.ops.append(eng.k_new[layer], eng.v_new[layer], eng.seq_lens[layer], eng.tail_idx, eng.pool[layer],
                           eng.block_table, eng.tail_k[layer], pos_offset=0, advance=True)
            if pg is not None:
                decode_gathered(eng.ops, eng.q[layer], eng.pool[layer], eng.block_table, eng.seq_lens[layer],
                                eng.tail_idx, eng.tail_k[layer], eng.scale, eng.ns, eng.work, pg,
                                parity * geo.L + layer)
                continue
            eng.ops.decode(eng.q[layer], eng.out[layer], eng.pool[layer], eng.block_table, eng.seq_lens[layer],
                           eng.tail_idx, eng.tail_k[layer], eng.scale, eng.ns, eng.work, fused=eng.fused)
            outs[layer].copy_(gather_heads(eng.out[layer]) if dist is not None else eng.out[layer])
        return out_sets[parity]

    def barrier():
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize(dev)

    steps_done = [0]                            # every rank runs the same sequence of steps, so parities agree

    def eager():
        steps_done[0] += 1
        return step((steps_done[0] - 1) % 2)

    for _ in range(a.warmup - 1):
        eager()
    graph = None
    if dist is None or pg is not None:          # the whole step as one CUDA graph (no library collective in it)
        graph = [capture(lambda: step(0), dev), capture(lambda: step(1), dev)]

        def run():
            p = steps_done[0] % 2
            steps_done[0] += 1
            graph[p].replay()
            return out_sets[p]
    else:                                       # NCCL collectives are never captured: eager steps
        run = eager
        eager()
    n0 = int(eng.seq_lens[0, 0].item())
    sampler = ClockSampler(local)               # started before the barrier: its spawn cannot skew the ranks
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(a.steps):
        run()
    e1.record()
    torch.cuda.synchronize(dev)
    clocks = sampler.stop()
    barrier()
    ms = e0.elapsed_time(e1)
    byts = sum(full.packed_bytes(n0 + i + 1) for i in range(a.steps)) * geo.L
    # ---- e2e: q and the new K/V rows of every layer from pinned host memory, every layer's (gathered) outputs back,
    # overlapped with the neighbouring steps (eager NCCL steps: copies around each step on the copy stream as well)
    io = OverlappedIO({k: getattr(eng, k) for k in ("q", "k_new", "v_new")}, out_sets[0], dev)
    io.run(1, run)
    n_e2e = int(eng.seq_lens[0, 0].item())
    barrier()
    x0, x1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    x0.record()
    io.run(a.steps, run)
    x1.record()
    torch.cuda.synchronize(dev)
    barrier()
    e2e_ms = x0.elapsed_time(x1)
    e2e_byts = sum(full.packed_bytes(n_e2e + i + 1) for i in range(a.steps)) * geo.L
    if dist is not None:
        t = torch.tensor([ms, e2e_ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, e2e_ms = (float(v) for v in t.tolist())
    if rank == 0:
        ms_step = ms / a.steps
        value = byts / (ms / 1e3) / 1e9
        print(json.dumps({
            "metric": METRIC, "value": round(value, 1), "unit": "GB/s", "n_gpus": world, "steps": a.steps,
            "warmup": a.warmup, "ms_per_step": round(ms_step, 4), "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "int4 records, bf16 q/k/v, fp32 softmax",
            "data": "synthetic (seeded bf16 N(0,1) K/V/q with per-channel key offsets N(0, 2), BASELINE config 4 shapes)",
            "config": {**full.describe(), "kv_heads_per_gpu": geo.HKV,
                       "parallelism": f"kv heads partitioned over {world} GPU(s), outputs "
                       "gathered per layer " + ("by the split-KV combine's stores into every rank's buffer over "
                       "NVLink (CUDA IPC), one wait kernel per layer" if pg is not None else
                       "by an NCCL all_gather" if dist is not None else "(one GPU: none)"), "n_splits": eng.ns,
                       "split_combine": "peer gather" if pg is not None else "fused" if eng.fused else "launch"},
            "pct_of_8TBs": round(100 * value / world / NOMINAL_HBM_GBS, 1),
            "us_per_layer_step": round(ms_step * 1e3 / geo.L, 2),
            "decode_tokens_per_s": round(geo.B / (ms_step / 1e3), 1), "clocks": clocks,
            "e2e": {"value": round(e2e_byts / (e2e_ms / 1e3) / 1e9, 1), "unit": "GB/s",
                    "h2d_bytes_per_step": io.h2d_bytes, "d2h_bytes_per_step": io.d2h_bytes,
                    "ms_per_step": round(e2e_ms / a.steps, 4)},
            "gpu_launches": a.steps * (eng.launches_per_step() + (geo.L if pg is not None else 0)),
            "cuda_graph": graph is not None}), flush=True)
    del graph, eng, io
    if pg is not None:
        pg.close()
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


# ---------------------------------------------------------------- ragged workloads: BASELINE configs 1, 2 and 5
MIX_SEQS, MIX_PROMPTS, MIX_PROMPT_LEN = 2048, 32, 2048


def mix_lengths(seed: int = 5) -> list[int]:
    """Context lengths of the 2048 decode sequences: lognormal, median 2048, sigma 0.8, capped at 16384 (seeded)."""
    gen = torch.Generator().manual_seed(seed)
    x = torch.randn(MIX_SEQS, generator=gen) * 0.8 + math.log(2048)
    return [int(min(16384, max(1, round(math.exp(v))))) for v in x.tolist()]


def offsets_qwen(hkv: int, D: int, gen: torch.Generator) -> torch.Tensor:
    """Configs 1 and 2: per kv head 4 of the 128 key channels offset by +-20 (random sign), the rest by N(0, 0.5)."""
    off = torch.randn(hkv, D, generator=gen) * 0.5
    for h in range(hkv):
        idx = torch.randperm(D, generator=gen)[:4]
        off[h, idx] = 20 * torch.sign(torch.randn(4, generator=gen))
    return off


def offsets_llama(hkv: int, D: int, gen: torch.Generator) -> torch.Tensor:
    """Configs 3 and 5: key offsets N(0, 2) plus 2 outlier channels at +-15 per kv head."""
    off = torch.randn(hkv, D, generator=gen) * 2
    for h in range(hkv):
        idx = torch.randperm(D, generator=gen)[:2]
        off[h, idx] = 15 * torch.sign(torch.randn(2, generator=gen))
    return off


def ragged_config(which: str, layers: int) -> dict:
    """The shapes of BASELINE configs 1 (c1), 2 (c2) and 5 (mix)."""
    if which == "c1":
        return dict(name="BASELINE config 1: Qwen2.5-7B attention geometry (28 q / 4 kv heads, head_dim 128), int4, "
                         "8 sequences x 2048 tokens written by quantize-on-write, page 32; one step = append + decode",
                    model="Qwen2.5-7B (attention geometry only)", hq=28, hkv=4, bits=4, P=32, lens=[2048] * 8,
                    prompts=0, layers=1, offsets=offsets_qwen, seed=0)
    if which == "c2":
        gen = torch.Generator().manual_seed(2)
        lens = torch.randint(256, 8193, (64,), generator=gen).tolist()
        return dict(name="BASELINE config 2: Qwen2.5-7B attention geometry, int8, 64 sequences with lengths "
                         "U[256, 8192], page 32; one step = append one token per sequence + decode",
                    model="Qwen2.5-7B (attention geometry only)", hq=28, hkv=4, bits=8, P=32, lens=lens, prompts=0,
                    layers=1, offsets=offsets_qwen, seed=2)
    return dict(name="BASELINE config 5: Llama-3.1-8B attention geometry, int4, page 16, 2048 sequences (lognormal "
                     "lengths, median 2048, sigma 0.8, cap 16384) + per step 32 prompts of 2048 tokens; "
                     f"{layers} of the 32 layers per step (all layers are the same work)",
                model="Llama-3.1-8B (attention geometry only: 32 q heads, 8 kv heads, head_dim 128)", hq=32, hkv=8,
                bits=4, P=16, lens=mix_lengths(), prompts=MIX_PROMPTS, layers=layers, offsets=offsets_llama, seed=5)


class RaggedEngine:
    """One GPU's share of a ragged workload: L layers of the decode sequences' caches, the pages of its share of the
    per-step prompts (config 5), and the per-step inputs.  keep_fill keeps layer 0's context K/V (one ragged write
    of every sequence) for the write roofline."""

    def __init__(self, cfg: dict, lens: list[int], n_prompts: int, device: torch.device, seed: int,
                 extra_tokens: int, keep_fill: bool, launch_order: str = "natural"):
        from kushkash_b200 import Ops
        self.dev, self.L, self.lens, self.PR = device, cfg["layers"], lens, n_prompts
        self.D, self.HKV, self.HQ, self.bits, self.P = 128, cfg["hkv"], cfg["hq"], cfg["bits"], cfg["P"]
        D, H, P, L = self.D, self.HKV, self.P, self.L
        self.DC = D // 2 if self.bits == 4 else D
        self.RB = 2 * P * self.DC + 4 * D + 4 * P
        self.ops = Ops(device, D, self.bits, self.HQ // H, torch.bfloat16, P)
        S = self.S = len(lens)
        gen = torch.Generator().manual_seed(seed)
        pages = torch.tensor([-(-(n + extra_tokens) // P) for n in lens], dtype=torch.int64)
        ppr = MIX_PROMPT_LEN // P
        n_blocks = int(pages.sum()) + n_prompts * ppr
        perm = torch.randperm(n_blocks, generator=gen).to(torch.int32)
        bt = torch.zeros(max(S, 1), int(pages.max()) if S else 1, dtype=torch.int32)
        o = 0
        for s, n in enumerate(pages.tolist()):
            bt[s, :n] = perm[o:o + n]
            o += n
        self.bt_dec = bt.to(device)
        self.bt_pr = perm[o:].view(n_prompts, ppr).to(device)
        self.pool = torch.zeros(L, n_blocks, H, self.RB, dtype=torch.uint8, device=device)
        self.tail_dec = torch.zeros(L, max(S, 1), H, P, D, dtype=torch.bfloat16, device=device)
        self.tail_pr = torch.zeros(L, max(n_prompts, 1), H, P, D, dtype=torch.bfloat16, device=device)
        self.ti_dec = torch.arange(max(S, 1), dtype=torch.int32, device=device)
        self.ti_pr = torch.arange(max(n_prompts, 1), dtype=torch.int32, device=device)
        self.sl_dec = torch.zeros(L, max(S, 1), dtype=torch.int32, device=device)
        self.sl_pr = torch.full((max(n_prompts, 1),), MIX_PROMPT_LEN, dtype=torch.int32, device=device)
        self.offsets = cfg["offsets"](H, D, gen).to(device)
        self.scale = 1.0 / math.sqrt(D)
        self.ns = self.ops.splits(S, H, max(lens) // P) if S else 1
        self.fused = FUSED_COMBINE
        self.work = torch.zeros(max(1, self.ops.work_size(max(S, 1), H, self.ns, self.fused)), device=device)
        dgen = torch.Generator(device=device).manual_seed(seed + 1)
        self.fill_in = None
        self._fill(dgen, keep_fill)
        self.sl_init = self.sl_dec.clone()
        T = n_prompts * MIX_PROMPT_LEN
        if n_prompts:
            self.pk = (torch.randn(L, T, H, D, generator=dgen, device=device) + self.offsets).to(torch.bfloat16)
            self.pv = torch.randn(L, T, H, D, generator=dgen, device=device).to(torch.bfloat16)
            self.pqsl = torch.arange(n_prompts + 1, dtype=torch.int32, device=device) * MIX_PROMPT_LEN
            self.pjs = torch.arange(n_prompts, dtype=torch.int32, device=device).repeat_interleave(ppr)
            self.pjp = torch.arange(ppr, dtype=torch.int32, device=device).repeat(n_prompts)
        self.k_new = (torch.randn(L, max(S, 1), H, D, generator=dgen, device=device) + self.offsets).to(torch.bfloat16)
        self.v_new = torch.randn(L, max(S, 1), H, D, generator=dgen, device=device).to(torch.bfloat16)
        self.q = torch.randn(L, max(S, 1), self.HQ, D, generator=dgen, device=device).to(torch.bfloat16)
        self.out = torch.empty_like(self.q)
        # longest-first decode launch order for ragged lengths over several waves of CTAs (computed once per step: the
        # layers share lengths); measured: config 5 (16k CTAs) step -4%, config 2 (512 CTAs, one wave) no gain
        self.order = None
        waves = S * H * self.ns / (4 * torch.cuda.get_device_properties(device).multi_processor_count)
        if launch_order == "longest" and S > 1 and min(lens) != max(lens) and waves > 2:
            self.order = torch.empty(S, dtype=torch.int32, device=device)

    def _jobs(self, seqs: list[int]):
        """Ragged write arguments for the whole contexts of `seqs`: query_start_loc over all S, job (seq, page)."""
        lens = torch.tensor(self.lens, dtype=torch.int64)
        rows = torch.zeros(self.S, dtype=torch.int64)
        rows[seqs] = lens[seqs]
        qsl = torch.cat([torch.zeros(1, dtype=torch.int64), rows.cumsum(0)]).to(torch.int32)
        npg = -(-lens[seqs] // self.P)
        js = torch.tensor(seqs, dtype=torch.int64).repeat_interleave(npg)
        start = torch.cat([torch.zeros(1, dtype=torch.int64), npg.cumsum(0)[:-1]]).repeat_interleave(npg)
        jp = torch.arange(int(npg.sum())) - start
        d = self.dev
        return qsl.to(d), js.to(torch.int32).to(d), jp.to(torch.int32).to(d), int(rows.sum())

    def _fill(self, dgen, keep: bool) -> None:
        """Bulk quantize-on-write of every decode sequence's context, per layer, in ragged chunks (one chunk when the
        inputs are kept)."""
        D, H = self.D, self.HKV
        limit = 1 << 62 if keep else 262144
        chunks, cur, tok = [], [], 0
        for s, n in enumerate(self.lens):
            if cur and tok + n > limit:
                chunks.append(cur)
                cur, tok = [], 0
            cur.append(s)
            tok += n
        if cur:
            chunks.append(cur)
        lens = torch.tensor(self.lens, dtype=torch.int32)
        for layer in range(self.L):
            for ch in chunks:
                qsl, js, jp, T = self._jobs(ch)
                k = (torch.randn(T, H, D, generator=dgen, device=self.dev) + self.offsets).to(torch.bfloat16)
                v = torch.randn(T, H, D, generator=dgen, device=self.dev).to(torch.bfloat16)
                self.sl_dec[layer, ch] = lens[ch].to(self.dev)
                self.ops.write(k, v, qsl, self.sl_dec[layer], self.ti_dec, js, jp, self.pool[layer], self.bt_dec,
                               self.tail_dec[layer])
                if keep and layer == 0:
                    self.fill_in = (k, v, qsl, js, jp)
        torch.cuda.synchronize(self.dev)

    def rewrite(self) -> None:
        """Layer 0's whole contexts again (the kept fill inputs), from the initial lengths."""
        k, v, qsl, js, jp = self.fill_in
        self.sl_dec[0].copy_(self.sl_init[0])
        self.ops.write(k, v, qsl, self.sl_dec[0], self.ti_dec, js, jp, self.pool[0], self.bt_dec, self.tail_dec[0])

    def prefill(self, layer: int) -> None:
        self.ops.write(self.pk[layer], self.pv[layer], self.pqsl, self.sl_pr, self.ti_pr, self.pjs, self.pjp,
                       self.pool[layer], self.bt_pr, self.tail_pr[layer])

    def decode(self, layer: int) -> None:
        self.ops.decode(self.q[layer], self.out[layer], self.pool[layer], self.bt_dec, self.sl_dec[layer], self.ti_dec,
                        self.tail_dec[layer], self.scale, self.ns, self.work, order=self.order, fused=self.fused)

    def step(self) -> None:
        """One step of every layer: the prompts' bulk prefill-quantize (config 5), append + decode of every sequence."""
        if self.order is not None:
            self.ops.longest_first(self.sl_dec[0], out=self.order)
        for layer in range(self.L):
            if self.PR:
                self.prefill(layer)
            if self.S:
                self.ops.append(self.k_new[layer], self.v_new[layer], self.sl_dec[layer], self.ti_dec,
                                self.pool[layer], self.bt_dec, self.tail_dec[layer], pos_offset=0, advance=True)
                self.decode(layer)

    def decode_bytes(self, extra: int, seqs: list[int] | None = None) -> int:
        """Packed-KV bytes of one decode layer-step with every sequence `extra` tokens past its initial length."""
        tot = 0
        for n in (self.lens if seqs is None else [self.lens[i] for i in seqs]):
            f, r = divmod(n + extra, self.P)
            tot += f * self.RB + r * (2 * self.D + self.DC + 4)
        return tot * self.HKV

    def io_bytes(self) -> int:
        """q in and out of one decode layer-step (bf16)."""
        return self.S * self.HQ * self.D * 4

    def prefill_bytes(self) -> int:
        """Algorithmic bytes of one layer's prompt write: bf16 K and V in, records out."""
        T = self.PR * MIX_PROMPT_LEN
        return 2 * T * self.HKV * self.D * 2 + (T // self.P) * self.HKV * self.RB

    def fill_bytes(self) -> int:
        """Algorithmic bytes of layer 0's whole-context write: bf16 K and V in, records (and partial pages' V rows
        and tail K rows) out."""
        T = sum(self.lens)
        return 2 * T * self.HKV * self.D * 2 + self.decode_bytes(0)

    def append_bytes(self) -> int:
        """Per layer: k, v rows in (bf16), the V code row and scale/bias and the exact K tail row out."""
        return self.S * self.HKV * (4 * self.D + self.DC + 4 + 2 * self.D)

    def launches_per_step(self) -> int:
        combine = 1 if self.ns > 1 and not self.fused else 0
        return (self.L * ((1 if self.PR else 0) + ((2 + combine) if self.S else 0))
                + (1 if self.order is not None else 0))


def time_graph(gr, dev, reps: int = 3) -> float:
    """ms per replay of a captured graph (one untimed replay first), CUDA events on the capture stream."""
    gr.replay()
    torch.cuda.synchronize(dev)
    k0, k1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    k0.record()
    for _ in range(reps):
        gr.replay()
    k1.record()
    torch.cuda.synchronize(dev)
    return k0.elapsed_time(k1) / reps


def time_cpu_ragged(cfg: dict, seqs: list[int], n_prompts: int, budget_s: float) -> dict:
    """The oracle on the host cores over a sample of a ragged workload (the given sequences at their lengths and
    n_prompts prompts): layer-steps of prompt write + append + decode until budget_s."""
    from oracle.kush_oracle import OracleOps, set_threads
    cores = set_threads(host_threads())
    D, H, P, bits, hq = 128, cfg["hkv"], cfg["P"], cfg["bits"], cfg["hq"]
    lens = [cfg["lens"][i] for i in seqs]
    gen = torch.Generator().manual_seed(99)
    off = cfg["offsets"](H, D, gen)
    ops = OracleOps(D, bits, hq // H, P)
    dc = D // 2 if bits == 4 else D
    rb = 2 * P * dc + 4 * D + 4 * P
    S = len(lens)
    max_iters = 2000                                    # every iteration appends one token per sequence: room for all
    pages = [-(-(n + max_iters + 8) // P) for n in lens]
    ppr = MIX_PROMPT_LEN // P
    nb = sum(pages) + n_prompts * ppr
    pool = torch.zeros(nb, H, rb, dtype=torch.uint8)
    perm = torch.randperm(nb, generator=gen).to(torch.int32)
    bt = torch.zeros(S, max(pages), dtype=torch.int32)
    o = 0
    for s, n in enumerate(pages):
        bt[s, :n] = perm[o:o + n]
        o += n
    bt_pr = perm[o:].view(n_prompts, ppr) if n_prompts else None
    tail = torch.zeros(S, H, P, D)
    ti = torch.arange(S, dtype=torch.int32)
    sl = torch.tensor(lens, dtype=torch.int32)
    T = sum(lens)
    k = (torch.randn(T, H, D, generator=gen) + off).bfloat16().float()
    v = torch.randn(T, H, D, generator=gen).bfloat16().float()
    qsl = torch.cat([torch.zeros(1, dtype=torch.int64), torch.tensor(lens).cumsum(0)]).to(torch.int32)
    npg = [-(-n // P) for n in lens]
    js = torch.tensor([s for s in range(S) for _ in range(npg[s])], dtype=torch.int32)
    jp = torch.tensor([p for s in range(S) for p in range(npg[s])], dtype=torch.int32)
    ops.write(k, v, qsl, sl, ti, js, jp, pool, bt, tail)
    q = torch.randn(S, hq, D, generator=gen).bfloat16().float()
    kn = (torch.randn(S, H, D, generator=gen) + off).bfloat16().float()
    vn = torch.randn(S, H, D, generator=gen).bfloat16().float()
    out = torch.empty_like(q)
    if n_prompts:
        pk = (torch.randn(n_prompts * MIX_PROMPT_LEN, H, D, generator=gen) + off).bfloat16().float()
        pv = torch.randn(n_prompts * MIX_PROMPT_LEN, H, D, generator=gen).bfloat16().float()
        pqsl = torch.arange(n_prompts + 1, dtype=torch.int32) * MIX_PROMPT_LEN
        psl = torch.full((n_prompts,), MIX_PROMPT_LEN, dtype=torch.int32)
        pti = torch.arange(n_prompts, dtype=torch.int32)
        ptail = torch.zeros(n_prompts, H, P, D)
        pjs = torch.arange(n_prompts, dtype=torch.int32).repeat_interleave(ppr)
        pjp = torch.arange(ppr, dtype=torch.int32).repeat(n_prompts)
    iters, byts, t0 = 0, 0, time.perf_counter()
    while True:
        if n_prompts:
            ops.write(pk, pv, pqsl, psl, pti, pjs, pjp, pool, bt_pr, ptail)
            byts += 2 * pk.numel() * 2 + (pk.shape[0] // P) * H * rb
        ops.append(kn, vn, sl, ti, pool, bt, tail, pos_offset=0, advance=True)
        ops.decode(q, out, pool, bt, sl, ti, tail, 1.0 / math.sqrt(D))
        byts += S * H * (4 * D + dc + 4 + 2 * D)
        for n in sl.tolist():
            f, r = divmod(n, P)
            byts += H * (f * rb + r * (2 * D + dc + 4))
        iters += 1
        el = time.perf_counter() - t0
        if el >= budget_s or iters >= max_iters:
            break
    return {"value": round(byts / el / 1e9, 3), "unit": "GB/s", "cores": cores, "kind": "port",
            "sample": f"{iters} layer-steps ({'prompt write + ' if n_prompts else ''}append + decode) of {S} of the "
                      f"{len(cfg['lens'])} sequences{f' and {n_prompts} of the prompts' if n_prompts else ''}, "
                      f"{el:.1f} s"}


def run_ragged(a, world: int, rank: int, local: int, which: str) -> None:
    """BASELINE configs 1 (c1), 2 (c2) and 5 (mix): ragged decode sequences (and, for config 5, per-step prompt bulk
    writes) with requests partitioned over the GPUs by tokens, no collective in the step.  Config 5's 32 layers of
    caches (~236 GB) do not fit one B200, so its step covers a subset of the layers (every layer is the same work)
    and its 32-layer figures are the measured layer-step time x 32."""
    from kushkash_b200.shard import partition_requests
    cfg = ragged_config(which, a.layers)
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist = None
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=300))
    lens_all = cfg["lens"]
    mine = partition_requests(lens_all, world)[rank]
    lens = [lens_all[i] for i in mine]
    n_pr = cfg["prompts"] // world
    eng = RaggedEngine(cfg, lens, n_pr, dev, seed=cfg["seed"] * 100 + rank, extra_tokens=a.warmup + 2 * a.steps + 8,
                       keep_fill=n_pr == 0, launch_order=a.launch_order)
    kern = {}
    if n_pr == 0:                                   # write roofline: layer 0's whole contexts again
        wgraph = capture(eng.rewrite, dev)
        kern["write"] = (eng.fill_bytes(), time_graph(wgraph, dev))
        del wgraph

    def barrier():
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize(dev)

    for _ in range(a.warmup - 1):
        eng.step()
    graph = capture(eng.step, dev)
    n_done = a.warmup - 1
    sampler = ClockSampler(local)               # started before the barrier: its spawn cannot skew the ranks
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(a.steps):
        graph.replay()
    e1.record()
    torch.cuda.synchronize(dev)
    clocks = sampler.stop()
    barrier()
    ms = e0.elapsed_time(e1)

    def step_bytes(first: int) -> int:
        b = sum(eng.decode_bytes(first + i + 1) for i in range(a.steps)) if eng.S else 0
        return (b + a.steps * (eng.prefill_bytes() * (1 if eng.PR else 0) + eng.append_bytes())) * eng.L

    byts = step_bytes(n_done)
    n_done += a.steps
    if eng.PR:
        wgraph = capture(lambda: [eng.prefill(l) for l in range(eng.L)], dev)
        kern["write"] = (eng.prefill_bytes(), time_graph(wgraph, dev) / eng.L)
        del wgraph
    if eng.S:
        dgraph = capture(lambda: [eng.decode(l) for l in range(eng.L)], dev)
        kern["decode"] = (eng.decode_bytes(n_done) + eng.io_bytes(), time_graph(dgraph, dev) / eng.L)
        del dgraph
    # e2e: every step's inputs (prompt K/V, new tokens, q) from pinned host memory, outputs back; steps of over 50 us
    # overlap each step's copies with its neighbours' kernels (OverlappedIO)
    # (short steps: the copies captured into the step's graph instead, CapturedIO)
    names = (("pk", "pv") if eng.PR else ()) + ("k_new", "v_new", "q")
    ins = {k: getattr(eng, k) for k in names}
    if ms / a.steps > 0.05:                        # measured: config 2 (108 us steps) gains from the overlap,
        io = OverlappedIO(ins, eng.out, dev)        # config 1 (24 us) is bound by the host work of it
    else:
        io = CapturedIO(ins, eng.out, dev, eng.step)
    io.run(1, graph.replay)
    n_done += 1
    barrier()
    x0, x1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    x0.record()
    io.run(a.steps, graph.replay)
    x1.record()
    torch.cuda.synchronize(dev)
    barrier()
    e2e_ms = x0.elapsed_time(x1)
    e2e_bytes = step_bytes(n_done)
    h2d, d2h = io.h2d_bytes, io.d2h_bytes
    if dist is not None:
        t = torch.tensor([ms, e2e_ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, e2e_ms = (float(x) for x in t.tolist())
        b = torch.tensor([float(byts), float(e2e_bytes)], device=dev, dtype=torch.float64)
        dist.all_reduce(b)
        byts, e2e_bytes = (float(x) for x in b.tolist())
    cpu = None
    if rank == 0 and world == 1 and not a.no_cpu_baseline:
        sample = list(range(len(lens_all))) if which != "mix" else list(range(16))
        cpu = time_cpu_ragged(cfg, sample, 1 if cfg["prompts"] else 0, a.cpu_seconds)
    if rank == 0:
        peak, peak_kind = hbm_peak()
        ms_step = ms / a.steps
        layer_us = ms_step * 1e3 / eng.L
        value = byts / (ms / 1e3) / 1e9
        roof = {}
        for name, (nb, kms) in kern.items():
            ach = nb / (kms / 1e3) / 1e9
            roof[name] = {"kernel": f"kush_sm100_{name}", "bound": "hbm", "achieved": round(ach, 1), "peak": peak,
                          "peak_kind": peak_kind, "unit": "GB/s", "frac": round(ach / peak, 4),
                          "algorithmic_bytes_per_launch": nb, "us_per_launch": round(kms * 1e3, 2), "rank": 0}
        S_all = len(lens_all)
        line = {
            "metric": METRIC, "value": round(value, 1), "unit": "GB/s", "n_gpus": world, "steps": a.steps,
            "warmup": a.warmup, "ms_per_step": round(ms_step, 4), "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": f"int{cfg['bits']} records, bf16 q/k/v, fp32 softmax",
            "data": f"synthetic (seeded bf16 N(0,1) K/V/q with per-channel key offsets; {cfg['name'].split(':')[0]} "
                    "shapes)",
            "config": {"workload": cfg["name"], "model": cfg["model"], "global_batch": S_all,
                       "cached_tokens": sum(lens_all), "layers_timed": eng.L, "page": cfg["P"], "bits": cfg["bits"],
                       "q_heads": cfg["hq"], "kv_heads": cfg["hkv"], "head_dim": 128,
                       "parallelism": f"requests partitioned over {world} GPU(s) by tokens, no collective in the step",
                       "launch_order": "longest first" if eng.order is not None else "natural",
                       "l2": ("inputs larger than L2 (GBs of records per layer-step, no flush needed)" if which == "mix"
                              else "inputs smaller than L2: the graph replays re-read L2-resident records (launch- "
                                   "and latency-bound sizes, as the config intends)")},
            "value_is": "all bytes of the step (decode packed-KV reads + appends" +
                        (" + prompt bf16 in / records out" if cfg["prompts"] else "") +
                        ") over the max-over-ranks device time",
            "per_gpu_gbs": round(value / world, 1),
            "pct_of_8TBs": round(100 * value / world / NOMINAL_HBM_GBS, 1),
            "us_per_layer_step": round(layer_us, 2),
            "e2e": {"value": round(e2e_bytes / (e2e_ms / 1e3) / 1e9, 1), "unit": "GB/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h, "ms_per_step": round(e2e_ms / a.steps, 4), "rank": 0},
            "roofline": roof.get("decode"), "write_roofline": roof.get("write"), "cpu_baseline": cpu,
            "clocks": clocks, "gpu_launches": a.steps * eng.launches_per_step(), "n_splits": eng.ns,
            "split_combine": "fused" if eng.fused else "launch"}
        if which == "mix":
            line["decode_tokens_per_s"] = round(S_all / (32 * layer_us / 1e6), 1)
            line["decode_tokens_per_s_is"] = ("2048 decode tokens per 32-layer step, the 32-layer step = 32 x the "
                                              "measured layer-step")
            line["prefill_tokens_per_s"] = round(MIX_PROMPTS * MIX_PROMPT_LEN / (32 * layer_us / 1e6), 1)
        else:
            line["decode_tokens_per_s"] = round(S_all / (ms_step / 1e3), 1)
            line["decode_tokens_per_s_is"] = "one layer (the config is a single-layer attention step)"
        print(json.dumps(line), flush=True)
    del graph, eng
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


# ---------------------------------------------------------------- unpack: prefill with history
UNPACK_METRIC = "unpack (prefill with history): algorithmic HBM GB/s"


class UnpackGeo:
    """The packed-prefill group of the vLLM / SGLang backends' prefill with history, per GPU and layer: S sequences
    of `hist` cached tokens -- full 16-token pages and a partial last page whose exact K sits in the tail slot -- and a
    new chunk of C rows each, unpacked by one launch into one [rows, 8, 128] workspace (the backends' ws.k / ws.v)."""

    def __init__(self, S: int = 32, hist: int = 4103, C: int = 512, L: int = 8):
        self.S, self.hist, self.C, self.L = S, hist, C, L
        self.D, self.H, self.P, self.bits = 128, 8, 16, 4
        self.DC = self.D // 2
        self.RB = 2 * self.P * self.DC + 4 * self.D + 4 * self.P
        self.fp, self.part = hist // self.P, hist % self.P
        self.npg = -(-hist // self.P)
        self.rows_per = hist + C

    def launch_bytes(self, S: int | None = None) -> int:
        """Algorithmic bytes of one layer's unpack over S sequences: full pages (record in, bf16 K and V rows out),
        the partial page (V code rows and scales, exact K rows in; K and V rows out), the new chunk (bf16 K and V in
        and out) and the int32 indices."""
        S = self.S if S is None else S
        H, D, P, part, C = self.H, self.D, self.P, self.part, self.C
        pages = self.fp * H * (self.RB + 2 * P * D * 2)
        partial = H * part * (self.DC + 4 + D * 2 + 2 * D * 2)
        new = C * H * D * 2 * 4
        return S * (pages + partial + new + 4 * (2 * self.fp + 4 + C))

    def indices(self, S: int) -> dict:
        """Host int32 unpack indices for S sequences with block table rows s * npg .. (identity table)."""
        fp, P = self.fp, self.P
        base = torch.arange(S, dtype=torch.int32) * self.rows_per
        bt = torch.arange(S * self.npg, dtype=torch.int32).view(S, self.npg)
        return {"page_blk": bt[:, :fp].reshape(-1).contiguous(),
                "page_dst": (base[:, None] + torch.arange(fp, dtype=torch.int32)[None] * P).reshape(-1).contiguous(),
                "tail_blk": bt[:, fp].contiguous(),
                "tail_info": torch.stack([base + fp * P, torch.full((S,), self.part, dtype=torch.int32),
                                          torch.arange(S, dtype=torch.int32)], 1).reshape(-1).contiguous(),
                "new_dst": (base[:, None] + self.hist + torch.arange(self.C, dtype=torch.int32)[None]).reshape(-1)
                .contiguous()}

    def describe(self) -> dict:
        return {"workload": f"prefill with history (unpack): Llama-3.1-8B kv geometry (8 kv heads, head_dim 128), "
                            f"int4, page 16; {self.S} sequences x {self.hist} cached tokens ({self.fp} full pages + a "
                            f"{self.part}-token partial page) + a {self.C}-row new chunk each, {self.L} layers per step",
                "model": "Llama-3.1-8B (attention geometry only)", "global_batch": self.S, "seq_len": self.rows_per,
                "layers": self.L,
                "l2": "inputs larger than L2 (%.2f GB of records and new rows per step)" % (
                    self.L * self.S * (self.npg * self.H * self.RB + 2 * self.C * self.H * self.D * 2) / 1e9)}


def unpack_jobs(geo: UnpackGeo, S: int):
    """Bulk-write arguments for S whole histories: query_start_loc, job (seq, page)."""
    qsl = torch.arange(S + 1, dtype=torch.int32) * geo.hist
    js = torch.arange(S, dtype=torch.int32).repeat_interleave(geo.npg)
    jp = torch.arange(geo.npg, dtype=torch.int32).repeat(S)
    return qsl, js, jp


class UnpackEngine:
    """One GPU's unpack workload: L layers of caches filled by the bulk quantize-on-write from seeded K / V, a seeded
    random block table, every layer's new rows, one shared output workspace."""

    def __init__(self, geo: UnpackGeo, device: torch.device, seed: int):
        from kushkash_b200 import Ops
        g = self.geo = geo
        S, H, D, P, L = g.S, g.H, g.D, g.P, g.L
        self.ops = Ops(device, D, g.bits, 4, torch.bfloat16, P)
        gen = torch.Generator().manual_seed(seed)
        dgen = torch.Generator(device=device).manual_seed(seed + 1)
        perm = torch.randperm(S * g.npg, generator=gen).to(torch.int32)
        bt = perm.view(S, g.npg)
        self.pool = torch.zeros(L, S * g.npg, H, g.RB, dtype=torch.uint8, device=device)
        self.tail = torch.zeros(L, S, H, P, D, dtype=torch.bfloat16, device=device)
        ti = torch.arange(S, dtype=torch.int32, device=device)
        offsets = offsets_llama(H, D, gen).to(device)
        qsl, js, jp = (x.to(device) for x in unpack_jobs(g, S))
        for layer in range(L):
            k = (torch.randn(S * g.hist, H, D, generator=dgen, device=device) + offsets).to(torch.bfloat16)
            v = torch.randn(S * g.hist, H, D, generator=dgen, device=device).to(torch.bfloat16)
            sl = torch.full((S,), g.hist, dtype=torch.int32, device=device)
            self.ops.write(k, v, qsl, sl, ti, js, jp, self.pool[layer], bt.to(device), self.tail[layer])
            del k, v
        idx = g.indices(S)
        idx["page_blk"] = bt[:, :g.fp].reshape(-1).contiguous()          # the random table's blocks
        idx["tail_blk"] = bt[:, g.fp].contiguous()
        self.idx = {k: v.to(device) for k, v in idx.items()}
        self.k_new = (torch.randn(L, S * g.C, H, D, generator=dgen, device=device) + offsets).to(torch.bfloat16)
        self.v_new = torch.randn(L, S * g.C, H, D, generator=dgen, device=device).to(torch.bfloat16)
        self.kp = torch.empty(S * g.rows_per, H, D, dtype=torch.bfloat16, device=device)
        self.vp = torch.empty_like(self.kp)
        torch.cuda.synchronize(device)

    def unpack(self, layer: int) -> None:
        x = self.idx
        self.ops.unpack(self.pool[layer], x["page_blk"], x["page_dst"], x["tail_blk"], x["tail_info"],
                        self.tail[layer], self.k_new[layer], self.v_new[layer], x["new_dst"], self.kp, self.vp,
                        rot=False)

    def step(self) -> None:
        for layer in range(self.geo.L):
            self.unpack(layer)


def time_cpu_unpack(geo: UnpackGeo, seqs: int, budget_s: float, min_calls: int = 1) -> dict:
    """The reference's CPU unpack (kushkash/kush/cpu.mojo:110-169, one thread; its C restatement in oracle/) over
    `seqs` sequences of one layer written by the oracle's bulk write, until budget_s; value in the same algorithmic
    bytes as the GPU figure."""
    from oracle.kush_oracle import OracleOps
    g = geo
    H, D, P = g.H, g.D, g.P
    gen = torch.Generator().manual_seed(99)
    ops = OracleOps(D, g.bits, 1, P)
    pool = torch.zeros(seqs * g.npg, H, g.RB, dtype=torch.uint8)
    tail = torch.zeros(seqs, H, P, D)
    off = offsets_llama(H, D, gen)
    qsl, js, jp = unpack_jobs(g, seqs)
    k = (torch.randn(seqs * g.hist, H, D, generator=gen) + off).bfloat16().float()
    v = torch.randn(seqs * g.hist, H, D, generator=gen).bfloat16().float()
    bt = torch.arange(seqs * g.npg, dtype=torch.int32).view(seqs, g.npg)
    ops.write(k, v, qsl, torch.full((seqs,), g.hist, dtype=torch.int32), torch.arange(seqs, dtype=torch.int32),
              js, jp, pool, bt, tail)
    x = g.indices(seqs)
    kn = (torch.randn(seqs * g.C, H, D, generator=gen) + off).bfloat16().float()
    vn = torch.randn(seqs * g.C, H, D, generator=gen).bfloat16().float()
    kp = torch.empty(seqs * g.rows_per, H, D)
    vp = torch.empty_like(kp)
    calls, t0 = 0, time.perf_counter()
    while True:
        ops.unpack(pool, x["page_blk"], x["page_dst"], x["tail_blk"], x["tail_info"], tail, kn, vn, x["new_dst"],
                   kp, vp, False)
        calls += 1
        el = time.perf_counter() - t0
        if calls >= min_calls and el >= budget_s:
            break
    return {"value": round(calls * g.launch_bytes(seqs) / el / 1e9, 3), "unit": "GB/s", "cores": 1, "kind": "port",
            "sample": f"{calls} unpacks of {seqs} of the {g.S} sequences (one layer), {el:.1f} s; fp32 output, bytes "
                      "counted as for the bf16 workload", "calls": calls, "seconds": el}


def unpack_traffic() -> float | None:
    """DRAM bytes per unpack launch at this workload from the committed ncu summary (profiles/), if present."""
    p = ROOT / "profiles" / "unpack_traffic.json"
    if p.exists():
        return float(json.loads(p.read_text())["total"])
    return None


def run_unpack(a, world: int, rank: int, local: int) -> None:
    """Prefill with history: K steps of L unpack launches (one CUDA graph per step); requests partitioned over the
    GPUs, no collective (weak scaling)."""
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist = None
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=120))
    geo = UnpackGeo(L=a.layers)
    eng = UnpackEngine(geo, dev, seed=77 + rank)

    def barrier():
        if dist is not None:
            dist.barrier()
        torch.cuda.synchronize(dev)

    for _ in range(a.warmup - 1):
        eng.step()
    graph = capture(eng.step, dev)
    graph.replay()
    sampler = ClockSampler(local)               # started before the barrier: its spawn cannot skew the ranks
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(a.steps):
        graph.replay()
    e1.record()
    torch.cuda.synchronize(dev)
    clocks = sampler.stop()
    barrier()
    ms = e0.elapsed_time(e1)
    # ---- e2e: the step's inputs (indices and every layer's new rows) from pinned host memory; back, the last packed
    # row of each sequence (K and V) -- the packed buffers themselves feed an attention kernel on the device
    hidx = {k: v.cpu().pin_memory() for k, v in eng.idx.items()}
    hk, hv = eng.k_new.cpu().pin_memory(), eng.v_new.cpu().pin_memory()
    last = torch.arange(1, geo.S + 1, device=dev) * geo.rows_per - 1
    hout = torch.empty(2, geo.S, geo.H, geo.D, dtype=torch.bfloat16).pin_memory()

    def e2e_step():
        for k_, t in hidx.items():
            eng.idx[k_].copy_(t, non_blocking=True)
        eng.k_new.copy_(hk, non_blocking=True)
        eng.v_new.copy_(hv, non_blocking=True)
        graph.replay()
        hout[0].copy_(eng.kp[last], non_blocking=True)
        hout[1].copy_(eng.vp[last], non_blocking=True)

    for _ in range(2):
        e2e_step()
    barrier()
    x0, x1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    x0.record()
    for _ in range(a.steps):
        e2e_step()
    x1.record()
    torch.cuda.synchronize(dev)
    barrier()
    e2e_ms = x0.elapsed_time(x1)
    h2d = sum(t.numel() * t.element_size() for t in hidx.values()) + 2 * hk.numel() * hk.element_size()
    d2h = hout.numel() * hout.element_size()
    if dist is not None:
        t = torch.tensor([ms, e2e_ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, e2e_ms = (float(v) for v in t.tolist())
    cpu = None
    if rank == 0 and world == 1 and not a.no_cpu_baseline:
        cpu = time_cpu_unpack(geo, 2, a.cpu_seconds)
        for k_ in ("calls", "seconds"):
            cpu.pop(k_)
    if rank == 0:
        peak, peak_kind = hbm_peak()
        step_bytes = geo.launch_bytes() * geo.L * world
        per_launch_ms = ms / (a.steps * geo.L)
        achieved = geo.launch_bytes() / (per_launch_ms / 1e3) / 1e9
        print(json.dumps({
            "metric": UNPACK_METRIC, "value": round(step_bytes * a.steps / (ms / 1e3) / 1e9, 1), "unit": "GB/s",
            "n_gpus": world, "steps": a.steps, "warmup": a.warmup, "ms_per_step": round(ms / a.steps, 4),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "int4 records, bf16 new rows and output, fp32 dequant",
            "data": "synthetic (seeded bf16 N(0,1) K/V with per-channel key offsets, written by the bulk write)",
            "config": {**geo.describe(), "parallelism": f"requests partitioned over {world} GPU(s), no collective"},
            "e2e": {"value": round(step_bytes * a.steps / (e2e_ms / 1e3) / 1e9, 1), "unit": "GB/s",
                    "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "ms_per_step": round(e2e_ms / a.steps, 4)},
            "roofline": {"kernel": "kush_sm100_unpack", "bound": "hbm", "achieved": round(achieved, 1), "peak": peak,
                         "peak_kind": f"{peak_kind} (HBM copy, MEASURED_PEAKS.json)" if peak_kind == "measured"
                         else "fallback", "unit": "GB/s", "frac": round(achieved / peak, 4),
                         "traffic": unpack_traffic(), "algorithmic_bytes_per_launch": geo.launch_bytes(),
                         "us_per_launch": round(per_launch_ms * 1e3, 2)},
            "cpu_baseline": cpu, "clocks": clocks, "gpu_launches": a.steps * geo.L}), flush=True)
    del graph, eng
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


def run_reference_unpack(a, world: int, rank: int) -> None:
    """The reference arm of the unpack workload: the reference's CPU unpack (one thread; its C restatement) on the
    host, each step one unpack of 2 of the sequences.  Rank 0 only."""
    if rank != 0:
        return
    from oracle.kush_oracle import build
    build()
    geo = UnpackGeo(L=a.layers)
    r = time_cpu_unpack(geo, 2, 0.0, min_calls=a.warmup)
    r = time_cpu_unpack(geo, 2, 0.0, min_calls=a.steps)
    value = r["value"]
    res = {"value": value, "unit": "GB/s", "cores": 1, "kind": "port",
           "sample": f"{a.steps} unpacks of 2 of the {geo.S} sequences (one layer), fp32 output"}
    print(json.dumps({"metric": UNPACK_METRIC, "value": value, "unit": "GB/s", "n_gpus": world, "steps": a.steps,
                      "warmup": a.warmup, "ms_per_step": round(r["seconds"] / r["calls"] * 1e3, 3),
                      "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
                      "dtype": "int4 records, fp32 compute", "impl": "reference", "data": "synthetic (seeded)",
                      "config": {**geo.describe(), "parallelism": "one host thread"}, "cpu_baseline": res,
                      "e2e": {"value": value, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}),
          flush=True)


def run_reference(a, geo: Geometry, world: int, rank: int) -> None:
    """The reference arm: the reference's CPU algorithm for this path (kushkash/kush/cpu.mojo, which needs the Mojo
    compiler that is not installed; timed through its C restatement in oracle/) on all host threads, each step one
    append + decode layer-step over a bounded sample of the workload.  Rank 0 only."""
    if rank != 0:
        return
    from oracle.kush_oracle import build
    build()
    seqs = min(a.cpu_seqs, geo.B)
    smp = cpu_sample_synthetic(geo, seqs, seed=1234, extra_tokens=a.warmup + a.steps + 8)
    for _ in range(a.warmup):
        time_cpu_decode(geo, smp, 0.0, with_append=True)
    res = time_cpu_decode(geo, smp, 0.0, with_append=True)
    t0 = time.perf_counter()
    byts = 0
    for _ in range(a.steps):
        r = time_cpu_decode(geo, smp, 0.0, with_append=True)
        byts += r["value"] * 1e9 * r["seconds_per_call"]
    el = time.perf_counter() - t0
    value = byts / el / 1e9
    res.update(value=round(value, 3), sample=f"{a.steps} layer-steps (append + decode) of {seqs} of the {geo.B} "
               f"sequences x {geo.HKV} kv heads at {geo.N}+ tokens, page {geo.P}, int4")
    res.pop("seconds_per_call", None)
    line = {"metric": METRIC, "value": round(value, 3), "unit": "GB/s", "n_gpus": world, "steps": a.steps,
            "warmup": a.warmup, "ms_per_step": round(el / a.steps * 1e3, 3), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "int4 records, fp32 compute", "impl": "reference",
            "data": "synthetic (seeded, BASELINE config 3 shapes)", "config": batch_config(geo, world),
            "reference_execution": f"host cores: the reference's CPU algorithm (its C restatement) with OpenMP over "
                                   f"(sequence, kv head) tasks on {res['cores']} threads, on a bounded sample of the "
                                   f"workload ({res['sample']})",
            "cpu_baseline": res,
            "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
