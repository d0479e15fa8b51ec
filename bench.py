#!/usr/bin/env python
"""Benchmark of the Q8_0 quantized linear hot path on B200.

Workload: the decode-step linear stack of a random-init
Qwen3-1.7B-shaped Q8_0 model at batch 1 - 28 layers of [qkv 4096x2048,
o 2048x2048, gate/up 12288x2048, down 2048x6144] plus the tied lm_head
151936x2048 - with int8 weights U[-127, 127] and fp16-drawn block scales
U[0.001, 0.01] widened to f32 (the reference's Q8 layout, 36 bytes per
block). One step is one token through all 113 projections. Dataflow per
layer: qkv reads the hidden state, o reads q (qkv rows 0..2047), gate/up
reads o's output, down reads gate (gate/up rows 0..6143); the lm_head reads
the last down output. Every layer's qkv reads the same hidden state x0: it
stands in for the RMSNorm output that feeds qkv in the real model (norms,
attention and SwiGLU are outside this hot path), and keeps the chained
activations finite. Stream order still serializes every projection.

Device path: x0 is quantized once per token (dn_quantize_qa); each GEMV
reads Q8_0-quantized activations and writes its outputs quantized again in
its epilogue (dn_linear_qa), so no projection re-quantizes on its own.

On N GPUs every matrix is split by output rows; each rank computes its row
slice and an NCCL all-gather over NVLink rebuilds the full activation for
the next projection (strong scaling: the model is fixed, rows are divided).
Outputs are bit-identical for every N: a row's result does not depend on the
split (lab_native.c:550-552).

Metric: tokens/s of the whole job (value), plus HBM GB/s of the weight
stream. `e2e` is the same token loop driven through the reference-facing
C-ABI with host activations and outputs: on one GPU through dianoia's
GPU-layer ABI (lab_gpu_*: one command buffer of 113 products per token, as
its GpuForward does); `e2e_cpu_abi` through the CPU-layer ABI (lab_gemm_q8,
one synchronous call per projection as NativeQ8Matrix.apply does), which is
also `e2e` on N > 1. `--impl reference`
times the reference's own CPU kernels (lab_native.c, compiled unmodified
into oracle/_ref) on this host's cores on the same workload.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import re
import os

# The host's cores as this process may use them, taken before any OpenMP
# runtime loads: a runtime started with a binding policy pins the main thread
# to one core, and the affinity read afterwards would say 1.
try:
    HOST_THREADS = len(os.sched_getaffinity(0))
except AttributeError:
    HOST_THREADS = os.cpu_count() or 1

import statistics
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

HIDDEN, HEADS, KV_HEADS, HEAD_DIM, INTER, LAYERS, VOCAB = 2048, 16, 8, 128, 6144, 28, 151936
# (name, rows, cols, input) per layer; qkv and gate/up are stored row-concatenated.
LAYER_MATS = [("qkv", (HEADS + 2 * KV_HEADS) * HEAD_DIM, HIDDEN),
              ("o", HEADS * HEAD_DIM, HEADS * HEAD_DIM),
              ("gate_up", 2 * INTER, HIDDEN),
              ("down", HIDDEN, INTER)]
Q8_BLOCK_BYTES_REF = 36   # reference layout: 32 int8 + f32 scale
Q8_BLOCK_BYTES_ALG = 34   # algorithmic credit: 32 int8 + fp16 scale (GGUF Q8_0)
METRIC = "quantized-linear HBM GB/s (GEMV), int8 TOPS (GEMM), tokens/s at 1/2/4/8 B200"
CHUNKS = 8                # weights are generated per 1/8 row chunk so any N in {1,2,4,8} shards alike
# DRAM bytes (read + write) of one GEMV launch per projection, from one ncu
# capture of each: a layer's four, and the lm_head.
MEASURED_DRAM_BYTES_LAYER = 9487872 + 4769024 + 28362496 + 14211072
MEASURED_DRAM_BYTES_HEAD = 350114304 + 4418560
# The chain kernel's DRAM bytes over reference-layout weight bytes, from one ncu
# capture of a 4-layer chain.
MEASURED_CHAIN_TRAFFIC_RATIO = (576637952 + 4725760) / 576552960


def log(*a):
    print(*a, file=sys.stderr, flush=True)


def set_layers(n: int) -> None:
    global LAYERS
    if n < 1:
        raise SystemExit("--layers must be >= 1")
    LAYERS = n


def matrices():
    """All projections of one token, in order: (layer, name, rows, cols)."""
    out = []
    for layer in range(LAYERS):
        for name, rows, cols in LAYER_MATS:
            out.append((layer, name, rows, cols))
    out.append((LAYERS, "lm_head", VOCAB, HIDDEN))
    return out


def step_bytes(block_bytes: int) -> int:
    """Weight + activation bytes one token must move through HBM."""
    total = 0
    for _, _, rows, cols in matrices():
        total += rows * (cols // 32) * block_bytes + cols * 4 + rows * 4
    return total


# ----------------------------------------------------------------- clocks

class ClockSampler:
    """nvidia-smi clocks and throttle reasons, sampled while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int):
        self.device_index = device_index
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.device_index}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
            time.sleep(0.3)
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc is not None:
            time.sleep(0.15)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax.append(float(parts[2]))
            except ValueError:
                continue
            for name, flag in zip(names, parts[5:9]):
                if flag.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": max(smax) if smax else None,
                "reasons": sorted(reasons), "samples": len(sm)}


# ------------------------------------------------------------------ model

def row_split(rows: int, rank: int, world: int, tiled: bool):
    """Rows [r0, r1) of a projection on `rank` of `world`: an even split, or,
    for the sharded chain, one on 32-row tiles (the chain's output unit)."""
    if not tiled:
        return rows * rank // world, rows * (rank + 1) // world
    tiles = -(-rows // 32)
    return min(rows, tiles * rank // world * 32), min(rows, tiles * (rank + 1) // world * 32)


def shard_rows(name: str, rows: int, rank: int, world: int, path: str):
    """Rows [r0, r1) of projection `name` on `rank` for a multi-GPU path:
    "chain" splits every projection on 32-row tiles, "ops" evenly, and
    "head" keeps the decoder layers whole on every GPU and splits only the
    lm_head's vocabulary rows (the reference's LM-head sharding,
    shard.dart:12-13), so a token crosses GPUs once, for its logits."""
    if path == "head" and name != "lm_head":
        return 0, rows
    return row_split(rows, rank, world, path == "chain")


def rank_bytes(mats, block_bytes: int) -> int:
    """Weight + activation bytes one rank moves per token for its row slices
    (the activation read in full, the slice's outputs written)."""
    return sum((m["r1"] - m["r0"]) * (m["cols"] // 32) * block_bytes + m["cols"] * 4
               + (m["r1"] - m["r0"]) * 4 for m in mats)


class Stack:
    """This rank's row slices of every projection, resident in HBM."""

    def __init__(self, torch, rank: int, world: int, device, path: str = "ops"):
        self.torch = torch
        self.rank, self.world, self.device = rank, world, device
        self.mats = []
        for idx, (layer, name, rows, cols) in enumerate(matrices()):
            r0, r1 = shard_rows(name, rows, rank, world, path)
            qs, sc = self._weights(idx, rows, cols, r0, r1)
            self.mats.append(dict(layer=layer, name=name, rows=rows, cols=cols, r0=r0, r1=r1,
                                  qs=qs, scales=sc))
        t = torch
        self.x0 = t.empty(HIDDEN, dtype=t.float32, device=device)
        gen = t.Generator(device=device)
        gen.manual_seed(12345)
        self.x0.normal_(generator=gen)
        self.bufs = {n: t.zeros(r, dtype=t.float32, device=device)
                     for n, r, _ in [("qkv", LAYER_MATS[0][1], 0), ("o", LAYER_MATS[1][1], 0),
                                     ("gate_up", LAYER_MATS[2][1], 0), ("down", HIDDEN, 0),
                                     ("lm_head", VOCAB, 0)]}

    def _weights(self, idx, rows, cols, r0, r1):
        t = self.torch
        blocks = cols // 32
        qs = t.empty((r1 - r0) * cols, dtype=t.int8, device=self.device)
        sc = t.empty((r1 - r0) * blocks, dtype=t.float32, device=self.device)
        step = rows // CHUNKS
        gen = t.Generator(device=self.device)
        for c in range(CHUNKS):
            c0, c1 = c * step, (c + 1) * step
            lo, hi = max(c0, r0), min(c1, r1)
            if lo >= hi:
                continue
            gen.manual_seed(1_000_003 * idx + c)
            chunk_q = t.randint(-127, 128, ((c1 - c0) * cols,), dtype=t.int8, device=self.device,
                                generator=gen)
            chunk_s = t.empty((c1 - c0) * blocks, dtype=t.float32, device=self.device)
            chunk_s.uniform_(0.001, 0.01, generator=gen)
            chunk_s = chunk_s.half().float()
            qs[(lo - r0) * cols:(hi - r0) * cols] = chunk_q[(lo - c0) * cols:(hi - c0) * cols]
            sc[(lo - r0) * blocks:(hi - r0) * blocks] = chunk_s[(lo - c0) * blocks:(hi - c0) * blocks]
        return qs, sc

    def input_name(self, m):
        """Which buffer feeds projection m (None: the hidden state x0)."""
        return {"qkv": None, "o": "qkv", "gate_up": "o", "down": "gate_up",
                "lm_head": "down"}[m["name"]]


INPUT_OF = {"qkv": None, "o": "qkv", "gate_up": "o", "down": "gate_up", "lm_head": "down"}
OUT_ROWS = {"qkv": LAYER_MATS[0][1], "o": LAYER_MATS[1][1], "gate_up": LAYER_MATS[2][1],
            "down": HIDDEN, "lm_head": VOCAB}


class QAChain:
    """Device buffers of the quantized-activation chain (QA blocks, 36 B per
    32 values) for one token."""

    def __init__(self, torch, device):
        self.xa0 = torch.zeros(HIDDEN // 32 * 36, dtype=torch.uint8, device=device)
        self.ya = {n: torch.zeros(r // 32 * 36, dtype=torch.uint8, device=device)
                   for n, r in OUT_ROWS.items() if n != "lm_head"}


def make_gather(dist, rank, world):
    """All-gather of a buffer whose rank p holds elements [numel * p // world,
    numel * (p + 1) // world) - the split of row_split, by elements - in place.
    An even split is one all_gather_into_tensor; otherwise each rank's span is
    padded to the widest span, gathered, and copied into place."""
    def gather(out):
        numel = out.numel()
        spans = [(numel * p // world, numel * (p + 1) // world) for p in range(world)]
        lo, hi = spans[rank]
        if numel % world == 0:
            dist.all_gather_into_tensor(out, out[lo:hi])
            return
        width = max(b - a for a, b in spans)
        send = out.new_zeros(width)
        send[:hi - lo] = out[lo:hi]
        recv = out.new_empty(world * width)
        dist.all_gather_into_tensor(recv, send)
        for p, (a, b) in enumerate(spans):
            out[a:b] = recv[p * width:p * width + b - a]
    return gather


class _DevArray:
    """A device f32 array at a raw address, for torch.as_tensor (no copy)."""

    def __init__(self, ptr, n):
        self.__cuda_array_interface__ = {"shape": (n,), "typestr": "<f4", "data": (ptr, False),
                                         "version": 3}


class FusedHead:
    """The head path's logits all-gather fused into the lm_head product
    (dn_linear_qa_allgather): every rank allocates one region (the whole
    logits, then a counter and the wait's expect word) that the others map
    (dn_peer_alloc / dn_peer_open); each rank's lm_head stores its vocabulary
    rows into every rank's logits over NVLink and counts its tiles in every
    rank's counter, and dn_peer_wait ends the token once all ranks' tiles are
    in. No NCCL call and no TMA touches peer memory."""

    def __init__(self, torch, stack, L, dist):
        from dianoia_b200 import _lib
        self.L, self.dist = L, dist
        rank, world = stack.rank, stack.world
        self.logits_bytes = VOCAB * 4
        self.region_bytes = (self.logits_bytes + 256 + 4095) // 4096 * 4096
        base = ctypes.c_void_p()
        handle = (ctypes.c_uint8 * _lib.DN_PEER_HANDLE_BYTES)()
        _lib.check(L.dn_peer_alloc(self.region_bytes, ctypes.byref(base), handle), "dn_peer_alloc")
        self.base = base.value
        handles = [None] * world
        dist.all_gather_object(handles, bytes(handle))
        self.opened, bases = [], []
        for p in range(world):
            if p == rank:
                bases.append(self.base)
                continue
            ptr = ctypes.c_void_p()
            h = (ctypes.c_uint8 * _lib.DN_PEER_HANDLE_BYTES).from_buffer_copy(handles[p])
            _lib.check(L.dn_peer_open(h, ctypes.byref(ptr)), "dn_peer_open")
            bases.append(ptr.value)
            self.opened.append(ptr.value)
        self.ys = (ctypes.c_void_p * world)(*bases)
        self.cnts = (ctypes.c_void_p * world)(*[b + self.logits_bytes for b in bases])
        self.counter = self.base + self.logits_bytes
        self.expect = self.base + self.logits_bytes + 4
        self.tiles = sum(-(-(r1 - r0) // 32) for r0, r1 in
                         (row_split(VOCAB, p, world, False) for p in range(world)))
        self.world = world
        self.logits = torch.as_tensor(_DevArray(self.base, VOCAB), device=stack.device)
        dist.barrier()  # every region mapped everywhere before any rank stores into it

    def lm_head(self, m, xa, stream_handle, flags):
        rc = self.L.dn_linear_qa_allgather(0, m["qs"].data_ptr(), m["scales"].data_ptr(), xa.data_ptr(),
                                           m["r1"] - m["r0"], m["cols"], m["r0"], self.ys, self.cnts,
                                           self.world, flags, stream_handle)
        if rc != 0:
            raise RuntimeError(f"dn_linear_qa_allgather failed: {self.L.dn_error_string(rc).decode()}")
        rc = self.L.dn_peer_wait(self.counter, self.expect, self.tiles, stream_handle)
        if rc != 0:
            raise RuntimeError(f"dn_peer_wait failed: {self.L.dn_error_string(rc).decode()}")

    def close(self):
        self.dist.barrier()  # no rank still stores into another's region
        for p in self.opened:
            self.L.dn_peer_close(p)
        self.opened = []
        self.dist.barrier()
        if self.base:
            self.L.dn_peer_free(self.base)
            self.base = None


def run_step(stack, chain, L, stream_handle, gather, gather_qa, flags=1, fused=None):
    """One token through all projections on `stream_handle`. Returns launches."""
    rc = L.dn_quantize_qa(stack.x0.data_ptr(), chain.xa0.data_ptr(), 1, HIDDEN,
                          HIDDEN // 32 * 36, stream_handle)
    if rc != 0:
        raise RuntimeError(f"dn_quantize_qa failed: {L.dn_error_string(rc).decode()}")
    launches = 1
    for m in stack.mats:
        name = m["name"]
        src = INPUT_OF[name]
        xa = chain.xa0 if src is None else chain.ya[src]
        out = stack.bufs[name]
        ya = chain.ya.get(name)
        rl = m["r1"] - m["r0"]
        if fused is not None and name == "lm_head":
            fused.lm_head(m, xa, stream_handle, flags)
            launches += 2
            continue
        rc = L.dn_linear_qa(0, m["qs"].data_ptr(), m["scales"].data_ptr(), xa.data_ptr(),
                            m["cols"] // 32 * 36, out.data_ptr() + 4 * m["r0"], rl,
                            None if ya is None else ya.data_ptr() + m["r0"] // 32 * 36,
                            0 if ya is None else OUT_ROWS[name] // 32 * 36,
                            rl, m["cols"], 1, flags, stream_handle)
        if rc != 0:
            raise RuntimeError(f"dn_linear_qa failed: {L.dn_error_string(rc).decode()}")
        launches += 1
        if gather is not None:
            if ya is None:
                gather(out)
            else:
                gather_qa(ya)
    return launches


class DecodeChain:
    """All projections of one token as ONE persistent kernel (dn_chain_run):
    weights stream without a gap between dependent projections. The chain
    keeps the model's order: each projection starts after the one before it
    (qkv after the previous layer's down), so no layer runs ahead of the
    last. Each op has its own QA output buffer; only the logits are kept in
    f32. One GPU only: the row shards of N > 1 need an all-gather between
    ops."""

    def __init__(self, torch, stack, qa, L, device):
        from dianoia_b200 import _lib
        self.L = L
        self.keep = []
        ops, last = [], {}
        for i, m in enumerate(stack.mats):
            name = m["name"]
            src = INPUT_OF[name]
            if src is not None:
                xa, dep = last[src]
            else:
                # qkv reads x0 (the stand-in for the norm output) but, as in the
                # model, starts only after the previous layer's down.
                xa, dep = qa.xa0.data_ptr(), (last["down"][1] if "down" in last else -1)
            ys = ya = None
            if name == "lm_head":
                ys = stack.bufs["lm_head"].data_ptr()
            else:
                buf = torch.zeros(m["rows"] // 32 * 36, dtype=torch.uint8, device=device)
                self.keep.append(buf)
                ya = buf.data_ptr()
                last[name] = (ya, i)
            ops.append(_lib.ChainOp(m["qs"].data_ptr(), m["scales"].data_ptr(), xa, ys, ya,
                                    m["rows"], m["cols"], dep))
        arr = (_lib.ChainOp * len(ops))(*ops)
        self.handle = ctypes.c_void_p()
        _lib.check(L.dn_chain_create(0, arr, len(ops), ctypes.byref(self.handle)), "dn_chain_create")

    def close(self):
        if self.handle:
            self.L.dn_chain_destroy(self.handle)
            self.handle = ctypes.c_void_p()


class ShardedChain:
    """N > 1: a token's projections as one chain kernel per GPU, each rank
    computing its row slices. A tile's QA output goes into every rank's copy
    of the output over NVLink and is counted in every rank's counters
    (dn_chain_create_sharded), so no collective runs between projections.
    Every rank maps every other rank's region (dn_peer_alloc / dn_peer_open);
    the logits stay rank-local (each rank its rows of the whole buffer)."""

    def __init__(self, torch, stack, qa, L, device, dist):
        from dianoia_b200 import _lib
        self.L, self.dist = L, dist
        rank, world = stack.rank, stack.world
        nops = len(stack.mats)
        offs, at = [], 0
        for m in stack.mats:
            if m["name"] == "lm_head":
                offs.append(None)
                continue
            offs.append(at)
            at = (at + m["rows"] // 32 * 36 + 15) // 16 * 16
        counters_off = at
        self.region_bytes = (at + 4 * (nops + 2) + 255) // 256 * 256
        base = ctypes.c_void_p()
        handle = (ctypes.c_uint8 * _lib.DN_PEER_HANDLE_BYTES)()
        _lib.check(L.dn_peer_alloc(self.region_bytes, ctypes.byref(base), handle), "dn_peer_alloc")
        self.base = base.value
        handles = [None] * world
        dist.all_gather_object(handles, bytes(handle))
        self.opened = []
        bases = (ctypes.c_void_p * world)()
        for p in range(world):
            if p == rank:
                bases[p] = self.base
                continue
            ptr = ctypes.c_void_p()
            h = (ctypes.c_uint8 * _lib.DN_PEER_HANDLE_BYTES).from_buffer_copy(handles[p])
            _lib.check(L.dn_peer_open(h, ctypes.byref(ptr)), "dn_peer_open")
            bases[p] = ptr.value
            self.opened.append(ptr.value)
        ops, row0, total, last = [], [], [], {}
        for i, m in enumerate(stack.mats):
            name = m["name"]
            src = INPUT_OF[name]
            if src is not None:
                xa, dep = last[src]
            else:
                xa, dep = qa.xa0.data_ptr(), (last["down"][1] if "down" in last else -1)
            ys = ya = None
            if name == "lm_head":
                ys = stack.bufs["lm_head"].data_ptr()
            else:
                ya = self.base + offs[i]
                last[name] = (ya, i)
            ops.append(_lib.ChainOp(m["qs"].data_ptr(), m["scales"].data_ptr(), xa, ys, ya,
                                    m["r1"] - m["r0"], m["cols"], dep))
            row0.append(m["r0"])
            total.append(m["rows"])
        arr = (_lib.ChainOp * nops)(*ops)
        self.handle = ctypes.c_void_p()
        _lib.check(L.dn_chain_create_sharded(0, arr, (ctypes.c_int64 * nops)(*row0),
                                             (ctypes.c_int64 * nops)(*total), nops, rank, world,
                                             bases, self.region_bytes, self.base + counters_off,
                                             ctypes.byref(self.handle)), "dn_chain_create_sharded")
        dist.barrier()  # every region mapped everywhere before any rank runs

    def close(self):
        if self.handle:
            self.L.dn_chain_destroy(self.handle)
            self.handle = ctypes.c_void_p()
        self.dist.barrier()  # no rank still writes into another's region
        for p in self.opened:
            self.L.dn_peer_close(p)
        self.opened = []
        self.dist.barrier()
        if self.base:
            self.L.dn_peer_free(self.base)
            self.base = None


class DecodeStack:
    """All projections of one token as ONE persistent kernel with one CTA per
    SM and every projection's rows split over all SMs (dn_stack_run). Each
    projection reads the f32 output of the one before it and quantizes it
    itself; qkv reads x0 after the previous layer's down, as in the model.
    Each op has its own f32 output buffer; the logits are stack.bufs
    ["lm_head"]. One GPU."""

    def __init__(self, torch, stack, L, device):
        from dianoia_b200 import _lib
        self.L = L
        self.keep = []
        ops, last = [], {}
        for i, m in enumerate(stack.mats):
            name = m["name"]
            src = INPUT_OF[name]
            if src is not None:
                x, dep = last[src]
            else:
                x, dep = stack.x0.data_ptr(), (last["down"][1] if "down" in last else -1)
            if name == "lm_head":
                y = stack.bufs["lm_head"].data_ptr()
            else:
                buf = torch.zeros(m["rows"], dtype=torch.float32, device=device)
                self.keep.append(buf)
                y = buf.data_ptr()
                last[name] = (y, i)
            ops.append(_lib.StackOp(m["qs"].data_ptr(), m["scales"].data_ptr(), x, y,
                                    m["rows"], m["cols"], dep))
        arr = (_lib.StackOp * len(ops))(*ops)
        self.handle = ctypes.c_void_p()
        _lib.check(L.dn_stack_create(0, arr, len(ops), ctypes.byref(self.handle)), "dn_stack_create")

    def run(self, stream_handle, flags=1):
        rc = self.L.dn_stack_run(self.handle, flags, stream_handle)
        if rc != 0:
            raise RuntimeError(f"dn_stack_run failed: {self.L.dn_error_string(rc).decode()}")
        return 1

    def close(self):
        if self.handle:
            self.L.dn_stack_destroy(self.handle)
            self.handle = ctypes.c_void_p()


def run_step_chain(stack, qa, dchain, L, stream_handle, flags=1):
    """One token: quantize x0, then every projection in one chain kernel."""
    rc = L.dn_quantize_qa(stack.x0.data_ptr(), qa.xa0.data_ptr(), 1, HIDDEN,
                          HIDDEN // 32 * 36, stream_handle)
    if rc != 0:
        raise RuntimeError(f"dn_quantize_qa failed: {L.dn_error_string(rc).decode()}")
    rc = L.dn_chain_run(dchain.handle, flags, stream_handle)
    if rc != 0:
        raise RuntimeError(f"dn_chain_run failed: {L.dn_error_string(rc).decode()}")
    return 2


# -------------------------------------------------------------- CPU legs

def host_weights(stack):
    return [(m["qs"].cpu().numpy(), m["scales"].cpu().numpy(), m["rows"], m["cols"])
            for m in stack.mats]


def cpu_reference_tokens(ref, hw, x0, threads: int, tokens: int):
    """Runs `tokens` decode steps of the stack through the reference's
    lab_gemm_q8 (mode 1) on the host; returns seconds per token and the logits."""
    maxc = max(c for _, _, _, c in hw)
    xq = np.zeros(maxc, np.int8)
    xsc = np.zeros(maxc // 32 + 1, np.float32)
    outs = {n: np.zeros(r, np.float32) for n, r in [("qkv", 4096), ("o", 2048), ("gate_up", 12288),
                                                   ("down", 2048), ("lm_head", VOCAB)]}
    names = [m[1] for m in matrices()]
    t0 = time.perf_counter()
    for _ in range(tokens):
        for (qs, sc, rows, cols), name in zip(hw, names):
            src = INPUT_OF[name]
            xin = x0 if src is None else np.ascontiguousarray(outs[src][:cols])
            ref.gemm("q8", qs, sc, xin, rows, cols, 1, mode=1, threads=threads,
                     out=(outs[name], xq, xsc))
    return (time.perf_counter() - t0) / tokens, outs["lm_head"].copy()


def cpu_model() -> str:
    """The host CPU's model name (/proc/cpuinfo), or the platform's processor string."""
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    import platform
    return platform.processor() or "unknown"


def host_threads():
    return HOST_THREADS


def bind_cpu_threads():
    """The reference CPU baseline runs under OpenMP with its threads pinned next
    to one another (OMP_PROC_BIND=close). The system libgomp that its library
    (and the oracle's) links reads this once, when it loads, so this is set
    just before the first of them loads - and not at startup, where torch's own
    OpenMP runtime would read it too and pin the main thread to one core."""
    os.environ.setdefault("OMP_PROC_BIND", "close")


def run_reference_arm(args, rank, world):
    """--impl reference: the reference's CPU kernels on this host's cores."""
    if rank != 0:
        return None
    from oracle import oracle as orc
    bind_cpu_threads()
    try:
        ref = orc.Reference()
    except FileNotFoundError as e:
        return {"impl": "reference", "unavailable": str(e)}
    rng = np.random.default_rng(0)
    # The same shapes and distributions as our arm; generated on the host.
    hw = []
    for _, _, rows, cols in matrices():
        qs, sc = orc.q8_weights(rng, rows, cols)
        hw.append((qs, sc, rows, cols))
    x0 = orc.activations(rng, 1, HIDDEN)
    threads = host_threads()
    for _ in range(args.warmup):
        cpu_reference_tokens(ref, hw, x0, threads, 1)
    times = []
    for _ in range(args.steps):
        s, _ = cpu_reference_tokens(ref, hw, x0, threads, 1)
        times.append(s)
    total = sum(times)
    value = args.steps / total
    return {
        "metric": METRIC, "value": value, "unit": "tokens/s", "impl": "reference",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1e3 * total / args.steps, "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": "int8", "data": "synthetic",
        "config": workload_config(),
        "parallelism": (f"the reference's CPU kernels on rank 0's host cores ({threads} threads); "
                        f"ranks 1..{world - 1} idle" if world > 1 else
                        f"the reference's CPU kernels on the host cores ({threads} threads)"),
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": threads, "kind": "reference",
                         "cpu_model": cpu_model(),
                         "omp_proc_bind": os.environ.get("OMP_PROC_BIND", "unset"),
                         "sample": f"{args.steps} full decode-step linear stacks (113 lab_gemm_q8 calls each)"},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "hbm_gbs": step_bytes(Q8_BLOCK_BYTES_REF) * value / 1e9,
    }


def workload_config():
    """The workload both arms run (the reference arm's line carries the same)."""
    return {"workload": "config3: Qwen3-1.7B-shaped Q8_0 decode-step linear stack, batch 1 "
                        "(28 x [qkv 4096x2048, o 2048x2048, gate/up 12288x2048, down 2048x6144] "
                        "+ lm_head 151936x2048)",
            "global_batch": 1, "layers": LAYERS,
            "weights_bytes_per_token_ref_layout": step_bytes(Q8_BLOCK_BYTES_REF),
            "l2": "inputs larger than L2 (1.94 GB of weights streamed per step)"}


def parallelism(world, path="ops", gather="fused"):
    """How this arm spreads the workload over the GPUs (a line's own key,
    outside `config`, which names the workload only)."""
    if world == 1:
        return "1 GPU"
    if path == "chain":
        return (f"row-sharded x{world}, every tile's QA output stored into the peers over NVLink "
                "inside the chain kernel")
    if path == "head":
        return (f"decoder layers replicated on each of {world} GPUs, lm_head vocabulary rows sharded "
                f"x{world}; the logits all-gathered " +
                ("inside the lm_head product (each rank's rows stored into every rank's logits over "
                 "NVLink, then a bounded wait on its counter)" if gather == "fused"
                 else "by one NCCL all-gather per token"))
    return f"row-sharded x{world} + NCCL all-gather per projection"


# ------------------------------------------------------------------ main

def main():
    ap = argparse.ArgumentParser(description=__doc__.split("\n")[0])
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=500)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-graph", action="store_true")
    ap.add_argument("--path", choices=["auto", "stack", "chain", "ops", "head"], default="auto",
                    help="stack: one persistent kernel per token, one CTA per SM, every "
                         "projection's rows split over all SMs (1 GPU); chain: one persistent kernel per token (on N > 1 GPUs with the "
                         "all-gather fused into it over NVLink); ops: one GEMV launch per "
                         "projection (N > 1: NCCL all-gather after each); head: the ops "
                         "launches with the decoder layers whole on every GPU and only the "
                         "lm_head's rows sharded (N > 1: one NCCL all-gather of the logits); "
                         "auto: ops on 1 GPU, head on N > 1")
    ap.add_argument("--gather", choices=["fused", "nccl"], default="fused",
                    help="head path on N > 1 GPUs: the logits all-gather fused into the lm_head "
                         "product (peer stores over NVLink), or one NCCL all-gather")
    ap.add_argument("--e2e-steps", type=int, default=50)
    ap.add_argument("--e2e-cpu-abi", action="store_true",
                    help="on N > 1 GPUs also time the per-projection lab_gemm_q8 loop")
    ap.add_argument("--neighbour-steps", type=int, default=30,
                    help="tokens of the decode stack with norms, SwiGLU and residual adds")
    ap.add_argument("--context", type=int, default=1024,
                    help="KV-cache position of the whole decode step (with attention)")
    ap.add_argument("--cpu-tokens", type=int, default=3)
    ap.add_argument("--sharded", action="store_true",
                    help="--workload configs: the row-sharded form (config 5 and the lm_head sweep), "
                         "also on one GPU (the N = 1 point of the same measurement)")
    ap.add_argument("--config-steps", type=int, default=50,
                    help="launches per case of the configs key (0: leave it out)")
    ap.add_argument("--workload", choices=["stack", "gemv", "gemm", "configs", "neighbours", "cache", "drain"],
                    default="stack",
                    help="stack: config 3 (the default bench line); gemv: one matrix "
                         "(configs 1, 2 and the lm_head M sweep; also the ncu case)")
    ap.add_argument("--cases", default="",
                    help="--workload configs on N > 1 GPUs (or --sharded): only the cases whose name matches "
                         "this regular expression")
    ap.add_argument("--fmt", choices=["q8", "q4"], default="q8")
    ap.add_argument("--gguf", action="store_true",
                    help="--workload gemv: the product on GGUF blocks as the file stores them (dn_gguf_linear_qa)")
    ap.add_argument("--rows", type=int, default=VOCAB)
    ap.add_argument("--cols", type=int, default=HIDDEN)
    ap.add_argument("--n", type=int, default=1, help="tokens per product")
    ap.add_argument("--layers", type=int, default=LAYERS,
                    help="decoder layers of the stack (28; fewer only for small profiler captures)")
    args = ap.parse_args()
    set_layers(args.layers)
    if args.workload == "gemv":
        return run_gemv_workload(args)
    if args.workload == "gemm":
        return run_gemm_workload(args)
    if args.workload == "configs":
        if int(os.environ.get("WORLD_SIZE", "1")) > 1 or args.sharded:
            return run_configs_sharded(args, int(os.environ.get("RANK", "0")),
                                       int(os.environ.get("WORLD_SIZE", "1")),
                                       int(os.environ.get("LOCAL_RANK", "0")))
        return run_configs_workload(args)
    if args.workload == "drain":
        return run_drain_workload(args)
    if args.workload == "neighbours":
        return run_neighbours_workload(args)
    if args.workload == "cache":
        return run_cache_workload(args)
    args.warmup = max(args.warmup, 3)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        res = run_reference_arm(args, rank, world)
        if rank == 0 and res is not None:
            print(json.dumps(res), flush=True)
        return

    import torch
    import torch.distributed as dist
    from datetime import timedelta

    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    if world > 1:
        # Keep stdout to the one JSON line: NCCL's own log lines (switched on
        # by the environment or an nccl.conf) go to stderr.
        os.environ.setdefault("NCCL_DEBUG_FILE", "/dev/stderr")
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=device)

    from dianoia_b200 import _lib
    L = _lib.lib()
    if L.lab_cpu_supported() != 1:
        raise SystemExit("no sm_100 device visible to libdianoia_b200")

    path = args.path if args.path != "auto" else ("ops" if world == 1 else "head")
    stack = Stack(torch, rank, world, device, path)
    torch.cuda.synchronize()

    chain = QAChain(torch, device)
    gather = gather_qa = None
    if world > 1:
        gather = make_gather(dist, rank, world)
        # The head path's layers are whole on every GPU: only the logits move.
        gather_qa = gather if path != "head" else (lambda ya: None)

    dchain = None
    if path == "chain":
        dchain = (DecodeChain(torch, stack, chain, L, device) if world == 1
                  else ShardedChain(torch, stack, chain, L, device, dist))
    fused = FusedHead(torch, stack, L, dist) if path == "head" and world > 1 and args.gather == "fused" else None
    if path == "stack" and world > 1:
        raise SystemExit("--path stack runs on one GPU")
    dstack = DecodeStack(torch, stack, L, device) if path == "stack" else None

    def one_step(handle):
        if dstack is not None:
            return dstack.run(handle)
        if dchain is not None:
            return run_step_chain(stack, chain, dchain, L, handle)
        return run_step(stack, chain, L, handle, gather, gather_qa, fused=fused)

    stream = torch.cuda.Stream(device=device)
    graph = None
    launches_per_step = (1 if dstack is not None else 2 if dchain is not None
                         else len(stack.mats) + 1 + (1 if fused is not None else 0))
    with torch.cuda.stream(stream):
        for _ in range(2):
            one_step(stream.cuda_stream)
        torch.cuda.synchronize()
        if not args.no_graph:
            try:
                graph = torch.cuda.CUDAGraph()
                with torch.cuda.graph(graph, stream=stream):
                    one_step(torch.cuda.current_stream().cuda_stream)
                torch.cuda.synchronize()
            except Exception as e:  # eager launches if capture is not possible
                log("graph capture failed, running eagerly:", repr(e))
                graph = None

    def step():
        if graph is not None:
            graph.replay()
        else:
            one_step(stream.cuda_stream)

    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()

    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    with ClockSampler(local_rank) as clocks:
        with torch.cuda.stream(stream):
            start.record(stream)
            for _ in range(args.steps):
                step()
            end.record(stream)
        torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    ms = start.elapsed_time(end)
    t = torch.tensor([ms], dtype=torch.float64, device=device)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_max = float(t.item())
    status = L.dn_device_status(1)
    if status != 0:
        raise SystemExit(f"kernel bounded wait timed out (status {status})")

    ms_per_step = ms_max / args.steps
    tokens_per_s = 1e3 / ms_per_step
    ref_bytes = step_bytes(Q8_BLOCK_BYTES_REF)

    # Dominant kernel: the fused quantize + GEMV launches (or the decode
    # chain). Achieved = algorithmic bytes per step / step time on the
    # launching stream (the activation quantize and any gaps included, so
    # this is a lower bound of the kernel's own bandwidth); on N GPUs, the
    # bytes of this rank's row slices.
    peaks = {}
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            peaks = json.load(f)
    except OSError:
        pass
    peak = float(peaks.get("hbm_gbs", 6650.0))
    per_rank_bytes = rank_bytes(stack.mats, Q8_BLOCK_BYTES_ALG)
    achieved = per_rank_bytes / (ms_per_step * 1e-3) / 1e9

    # Checksum of the logits: identical for every N (rows do not depend on the
    # split). The sharded chain leaves each rank its own rows of the logits
    # (the rest zero): a sum over ranks rebuilds them exactly.
    full_logits = (fused.logits if fused is not None else stack.bufs["lm_head"]).clone()
    if world > 1 and dchain is not None:
        dist.all_reduce(full_logits)
    checksum = float(full_logits.double().sum().item())
    chain_matches_ops = None
    if (dchain is not None or dstack is not None) and world == 1:
        # The chain's logits equal the per-projection launches', bit for bit.
        chain_logits = stack.bufs["lm_head"].clone()
        with torch.cuda.stream(stream):
            stack.bufs["lm_head"].fill_(float("nan"))
            run_step(stack, chain, L, stream.cuda_stream, None, None)
        torch.cuda.synchronize()
        chain_matches_ops = bool(torch.equal(chain_logits.view(torch.int32),
                                             stack.bufs["lm_head"].view(torch.int32)))

    # End to end with host buffers: on one GPU through dianoia's GPU-layer
    # ABI (one command buffer per token); also, and on N > 1 only, through
    # the CPU-layer ABI (lab_gemm_q8 per projection on rank-local shards, the
    # slices all-gathered through device copies).
    e2e_cpu_abi = run_e2e(args, stack, L, torch, rank, world, gather, device, full_logits) \
        if world == 1 or args.e2e_cpu_abi else None
    e2e_dn = run_e2e_device_api(args, torch, stack, step, stream,
                                fused.logits if fused is not None else stack.bufs["lm_head"], world, device,
                                full_logits) if dchain is None else None
    e2e = run_e2e_gpu_layer(args, stack, L, torch) if world == 1 else None
    if e2e is None:
        e2e = e2e_dn if e2e_dn is not None else e2e_cpu_abi
    neighbours = run_neighbours(args, stack, L) if world == 1 else None
    decode_step = run_neighbours(args, stack, L, context=args.context) if world == 1 else None

    cpu_baseline = None
    if rank == 0 and world == 1 and args.cpu_tokens > 0:
        cpu_baseline = run_cpu_baseline(args, stack)
    configs = None
    if rank == 0 and world == 1 and args.config_steps > 0:
        configs = run_configs_compact(args, torch, L)

    if rank == 0:
        res = {
            "metric": METRIC, "value": tokens_per_s, "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_per_step,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "int8",
            "data": "synthetic (random-init Q8_0 weights, N(0,1) activations, seeded)",
            "config": workload_config(),
            "parallelism": parallelism(world, path, args.gather),
            "hbm_gbs_per_gpu": rank_bytes(stack.mats, Q8_BLOCK_BYTES_REF) / (ms_per_step * 1e-3) / 1e9,
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak,
                         "peak_source": "MEASURED_PEAKS.json hbm_gbs" if peaks else "fallback 6650",
                         "algorithmic_bytes_per_step_per_gpu": per_rank_bytes,
                         "traffic": (LAYERS * MEASURED_DRAM_BYTES_LAYER + MEASURED_DRAM_BYTES_HEAD / world
                                     if dchain is None and path == "head" else
                                     (LAYERS * MEASURED_DRAM_BYTES_LAYER + MEASURED_DRAM_BYTES_HEAD) / world
                                     if dchain is None else MEASURED_CHAIN_TRAFFIC_RATIO * ref_bytes / world),
                         "traffic_source": ("ncu per-launch DRAM bytes (read + write) of each "
                                            "projection's GEMV, summed per token" +
                                            (", the lm_head's / N" if path == "head" else ", / N")
                                            if dchain is None
                                            else "ncu DRAM bytes of a 4-layer chain launch, scaled "
                                                 "by weight bytes")},
            "e2e": e2e,
            "e2e_cpu_abi": e2e_cpu_abi,
            "e2e_device_api": e2e_dn,
            "neighbours": neighbours,
            "decode_step": decode_step,
            "cpu_baseline": cpu_baseline,
            "configs": configs,
            "gpu_launches": launches_per_step * args.steps,
            "gpu_launches_note": ("1 decode-stack kernel (113 products, each quantizing its f32 input) per step"
                                  if dstack is not None else
                                  "1 activation quantize + 1 decode-chain kernel (113 fused GEMVs) per step"
                                  if dchain is not None else
                                  "1 activation quantize + 113 fused GEMVs per step"),
            "path": path,
            "chain_logits_match_per_op_launches": chain_matches_ops,
            "graph": graph is not None,
            "clocks": clocks.summary(),
            "logits_checksum": checksum,
        }
        print(json.dumps(res), flush=True)
    graph = None  # graphs holding NCCL calls go before the process group
    torch.cuda.synchronize()
    if dchain is not None:
        dchain.close()
    if dstack is not None:
        dstack.close()
    if fused is not None:
        fused.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def run_gemv_workload(args):
    """One quantized matrix times n tokens through dn_linear_qa, timed with CUDA
    events on the launching stream; the weights rotate through enough copies
    to exceed twice the L2, so every launch streams them from HBM."""
    import torch
    from dianoia_b200 import _lib
    L = _lib.lib()
    rows, cols, n, q4 = args.rows, args.cols, args.n, args.fmt == "q4"
    blocks = cols // 32
    gguf = args.gguf
    if gguf and n != 1:
        raise SystemExit("--gguf runs one token")
    wbytes = rows * blocks * ((18 if q4 else 34) if gguf else (18 if q4 else 36))
    l2 = torch.cuda.get_device_properties(0).L2_cache_size
    copies = max(1, -(-2 * l2 // wbytes))
    gen = torch.Generator(device="cuda")
    gen.manual_seed(0)
    mats = []
    for _ in range(copies):
        if gguf:
            mats.append((gguf_device_blocks(torch, args.fmt, rows, cols, gen), None))
            continue
        if q4:
            qs = torch.randint(0, 256, (rows * cols // 2,), dtype=torch.uint8, device="cuda", generator=gen)
            sc = torch.empty(rows * blocks, device="cuda").uniform_(0.002, 0.02, generator=gen)
            sc = sc.half().view(torch.int16)
        else:
            qs = torch.randint(-127, 128, (rows * cols,), dtype=torch.int8, device="cuda", generator=gen)
            sc = torch.empty(rows * blocks, device="cuda").uniform_(0.001, 0.01, generator=gen)
            sc = sc.half().float()
        mats.append((qs, sc))
    x = torch.randn(n * cols, device="cuda", generator=gen)
    xa = torch.zeros(n * blocks * 36, dtype=torch.uint8, device="cuda")
    ys = torch.zeros(n * rows, device="cuda")
    ya = torch.zeros(n * (rows // 32) * 36, dtype=torch.uint8, device="cuda")
    stream = torch.cuda.Stream()
    h = stream.cuda_stream
    assert L.dn_quantize_qa(x.data_ptr(), xa.data_ptr(), n, cols, blocks * 36, h) == 0

    def launch(i, handle):
        qs, sc = mats[i % copies]
        if gguf:
            rc = L.dn_gguf_linear_qa(1 if q4 else 0, qs.data_ptr(), xa.data_ptr(), ys.data_ptr(), rows, cols, 1,
                                     handle)
        else:
            rc = L.dn_linear_qa(1 if q4 else 0, qs.data_ptr(), sc.data_ptr(), xa.data_ptr(),
                                blocks * 36, ys.data_ptr(), rows, ya.data_ptr(), (rows // 32) * 36,
                                rows, cols, n, 1, handle)
        if rc != 0:
            raise RuntimeError(L.dn_error_string(rc).decode())

    with torch.cuda.stream(stream):
        for i in range(max(args.warmup, 1)):
            launch(i, h)
        torch.cuda.synchronize()
        graph = None
        if not args.no_graph:
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=stream):
                for i in range(args.steps):
                    launch(i, torch.cuda.current_stream().cuda_stream)
            graph.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        if graph is not None:
            graph.replay()
        else:
            for i in range(args.steps):
                launch(i, h)
        e1.record(stream)
        torch.cuda.synchronize()
    if L.dn_device_status(1) != 0:
        raise SystemExit("kernel bounded wait timed out")
    us = e0.elapsed_time(e1) * 1e3 / args.steps
    alg = rows * blocks * (18 if q4 else 34) + n * cols * 4 + n * rows * 4
    peaks = {}
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            peaks = json.load(f)
    except OSError:
        pass
    peak = float(peaks.get("hbm_gbs", 6650.0))
    res = {"metric": "quantized-linear GEMV HBM GB/s",
           "workload": f"{args.fmt} {rows}x{cols} n={n}" + (" (GGUF blocks as stored)" if gguf else ""),
           "us_per_launch": us, "weight_bytes_ref_layout": wbytes,
           "gbs_ref_layout": wbytes / us / 1e3, "gbs_algorithmic": alg / us / 1e3,
           "roofline_frac": alg / us / 1e3 / peak, "peak_gbs": peak, "copies": copies,
           "launches": args.steps, "graph": graph is not None,
           "l2": f"{copies} rotating weight copies (> 2 x L2)"}
    print(json.dumps(res), flush=True)


def run_gemm_workload(args):
    """One quantized matrix times n tokens through dn_linear (tensor-core path
    when n is above the crossover): activation quantize + GEMM per launch,
    timed with CUDA events; reports int8 TOPS (2 * n * rows * cols per launch).
    Weights, activations and outputs rotate through enough copies to exceed
    twice the L2, so each launch reads its operands from HBM."""
    import torch
    from dianoia_b200 import _lib
    L = _lib.lib()
    rows, cols, n, q4 = args.rows, args.cols, args.n, args.fmt == "q4"
    blocks = cols // 32
    gen = torch.Generator(device="cuda")
    gen.manual_seed(0)
    per_copy = rows * cols // (2 if q4 else 1) + rows * blocks * (2 if q4 else 4) + 4 * n * (cols + rows)
    l2 = torch.cuda.get_device_properties(0).L2_cache_size
    copies = max(1, -(-2 * l2 // per_copy))
    sets = []
    for _ in range(copies):
        if q4:
            qs = torch.randint(0, 256, (rows * cols // 2,), dtype=torch.uint8, device="cuda", generator=gen)
            sc = torch.empty(rows * blocks, device="cuda").uniform_(0.002, 0.02, generator=gen).half().view(torch.int16)
        else:
            qs = torch.randint(-127, 128, (rows * cols,), dtype=torch.int8, device="cuda", generator=gen)
            sc = torch.empty(rows * blocks, device="cuda").uniform_(0.001, 0.01, generator=gen).half().float()
        xs = torch.randn(n * cols, device="cuda", generator=gen)
        ys = torch.zeros(n * rows, device="cuda")
        sets.append((qs, sc, xs, ys))
    xq = torch.zeros(n * cols, dtype=torch.int8, device="cuda")
    xsc = torch.zeros(n * blocks + 4, device="cuda")
    stream = torch.cuda.Stream()
    qs0, sc0, xs0, _ = sets[0]
    path = L.dn_linear_path(1 if q4 else 0, qs0.data_ptr(), sc0.data_ptr(), xs0.data_ptr(),
                            xq.data_ptr(), rows, cols, n, 1)

    def launch(i, handle):
        qs, sc, xs, ys = sets[i % copies]
        rc = L.dn_linear(1 if q4 else 0, qs.data_ptr(), sc.data_ptr(), xs.data_ptr(), xq.data_ptr(),
                         xsc.data_ptr(), ys.data_ptr(), rows, cols, n, rows, 1, -1, 0, handle)
        if rc != 0:
            raise RuntimeError(L.dn_error_string(rc).decode())

    with torch.cuda.stream(stream):
        for i in range(max(args.warmup, 1)):
            launch(i, stream.cuda_stream)
        torch.cuda.synchronize()
        graph = None
        if not args.no_graph:
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=stream):
                for i in range(args.steps):
                    launch(i, torch.cuda.current_stream().cuda_stream)
            graph.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        if graph is not None:
            graph.replay()
        else:
            for i in range(args.steps):
                launch(i, stream.cuda_stream)
        e1.record(stream)
        torch.cuda.synchronize()
    if L.dn_device_status(1) != 0:
        raise SystemExit("kernel bounded wait timed out")
    us = e0.elapsed_time(e1) * 1e3 / args.steps
    ops = 2.0 * n * rows * cols
    peaks = {}
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            peaks = json.load(f)
    except OSError:
        pass
    # int8 dense tensor peak: twice the measured bf16 dense figure (the
    # nominal ratio, 4.5 vs 2.25 PFLOP/s).
    int8_peak = 2.0 * float(peaks.get("bf16_tflops", 1590.0))
    res = {"metric": "quantized-linear int8 GEMM TOPS", "workload": f"{args.fmt} {rows}x{cols} n={n}",
           "path": {0: "gemv", 1: "tcgen05", 2: "generic"}.get(path, path),
           "us_per_launch": us, "tops": ops / us / 1e6, "int8_peak_tops": int8_peak,
           "frac_of_int8_peak": ops / us / 1e6 / int8_peak,
           "peak_source": "2 x MEASURED_PEAKS.json bf16_tflops" if peaks else "2 x fallback 1590",
           "launches": args.steps, "graph": graph is not None, "copies": copies,
           "l2": f"{copies} rotating operand copies (> 2 x L2)",
           "includes": "activation quantize (f32 -> Q8_0) + GEMM"}
    print(json.dumps(res), flush=True)


# BASELINE configs 1, 2, 4, 5 and the lm_head M sweep: (config, name, fmt, rows, cols, n).
CONFIG_CASES = (
    [("c1", "mlp_up", "q4", 6144, 2048, 1)]
    + [("c2", n, "q8", r, c, 1) for n, r, c in [("q", 2048, 2048), ("k", 1024, 2048), ("v", 1024, 2048),
                                               ("o", 2048, 2048), ("gate", 6144, 2048),
                                               ("up", 6144, 2048), ("down", 2048, 6144)]]
    + [("c4", n, "q4", r, c, 512) for n, r, c in [("gate_up", 6144, 2048), ("down", 2048, 6144)]]
    # vision encoder, 1024 tokens; fc2's K 4304 padded to 4320 (a multiple of the 32-block)
    + [("c5", n, "q8", r, c, 1024) for n, r, c in [("qkv", 3456, 1152), ("o", 1152, 1152),
                                                   ("fc1", 4304, 1152), ("fc2", 1152, 4320)]]
    + [("c5", f"lm_head_m{m}", "q8", VOCAB, HIDDEN, m) for m in (1, 2, 4, 8, 16, 32, 64)])


def device_weights(torch, L, fmt, rows, cols, gen, vision=False):
    """One matrix of a configuration on the device: Q4_0 nibbles U{0..15} with
    fp16 scales U[0.002, 0.02] (config 1 / 4), Q8_0 int8 U[-127, 127] with
    fp16-drawn scales U[0.001, 0.01] widened to f32 (config 2 / 3 / lm_head),
    or config 5's: bf16 N(0, 0.02) weights quantized to Q8_0 on the device
    with lab_quantize_q8 semantics (dn_quantize_q8)."""
    blocks = cols // 32
    if fmt == "q4":
        qs = torch.randint(0, 256, (rows * cols // 2,), dtype=torch.uint8, device="cuda", generator=gen)
        sc = torch.empty(rows * blocks, device="cuda").uniform_(0.002, 0.02, generator=gen).half().view(torch.int16)
        return qs, sc
    if vision:
        w = (torch.randn(rows * cols, device="cuda", generator=gen) * 0.02).bfloat16().float()
        qs = torch.empty(rows * cols, dtype=torch.int8, device="cuda")
        sc = torch.empty(rows * blocks, dtype=torch.float32, device="cuda")
        rc = L.dn_quantize_q8(w.data_ptr(), qs.data_ptr(), sc.data_ptr(), rows, cols,
                              torch.cuda.current_stream().cuda_stream)
        if rc != 0:
            raise RuntimeError(L.dn_error_string(rc).decode())
        return qs, sc
    qs = torch.randint(-127, 128, (rows * cols,), dtype=torch.int8, device="cuda", generator=gen)
    sc = torch.empty(rows * blocks, device="cuda").uniform_(0.001, 0.01, generator=gen).half().float()
    return qs, sc


def time_linear(torch, L, fmt, rows, cols, n, steps, warmup, vision=False):
    """us per dn_linear launch (mode 1, automatic path, f32 activations in),
    the operands rotating through copies that exceed twice the L2 (weights
    generated once and copied)."""
    q4 = fmt == "q4"
    blocks = cols // 32
    per_copy = rows * cols // (2 if q4 else 1) + rows * blocks * (2 if q4 else 4) + 4 * n * (cols + rows)
    l2 = torch.cuda.get_device_properties(0).L2_cache_size
    copies = max(1, -(-2 * l2 // per_copy))
    gen = torch.Generator(device="cuda")
    gen.manual_seed(rows * 31 + cols * 7 + n)
    qs0, sc0 = device_weights(torch, L, fmt, rows, cols, gen, vision)
    sets = []
    for i in range(copies):
        qs, sc = (qs0, sc0) if i == 0 else (qs0.clone(), sc0.clone())
        sets.append((qs, sc, torch.randn(n * cols, device="cuda", generator=gen),
                     torch.zeros(n * rows, device="cuda")))
    xq = torch.zeros(n * cols, dtype=torch.int8, device="cuda")
    xsc = torch.zeros(n * blocks + 4, device="cuda")
    path = L.dn_linear_path(1 if q4 else 0, sets[0][0].data_ptr(), sets[0][1].data_ptr(),
                            sets[0][2].data_ptr(), xq.data_ptr(), rows, cols, n, 1)
    stream = torch.cuda.Stream()

    def launch(i, h):
        qs, sc, xs, ys = sets[i % copies]
        rc = L.dn_linear(1 if q4 else 0, qs.data_ptr(), sc.data_ptr(), xs.data_ptr(), xq.data_ptr(),
                         xsc.data_ptr(), ys.data_ptr(), rows, cols, n, rows, 1, -1, 1, h)
        if rc != 0:
            raise RuntimeError(L.dn_error_string(rc).decode())

    with torch.cuda.stream(stream):
        for i in range(warmup):
            launch(i, stream.cuda_stream)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            for i in range(steps):
                launch(i, torch.cuda.current_stream().cuda_stream)
        graph.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        graph.replay()
        e1.record(stream)
        torch.cuda.synchronize()
    del graph
    if L.dn_device_status(1) != 0:
        raise SystemExit("kernel bounded wait timed out")
    return e0.elapsed_time(e1) * 1e3 / steps, {0: "gemv", 1: "tcgen05", 2: "generic"}.get(path, path), copies


CHECK_ROWS = 512  # rows of a case's output checked against the oracle


def check_linear(torch, L, oracle, fmt, rows, cols, n, vision=False):
    """One dn_linear launch (mode 1, automatic path) on seeded inputs, its
    first CHECK_ROWS rows against the oracle (a row depends only on its own
    weights): bit for bit on the GEMV, within the reference's 1e-5 bound of
    the row's absolute-sum scale on the tensor-core GEMM. Returns (path, ok,
    max relative error)."""
    from oracle import oracle as orc
    q4 = fmt == "q4"
    blocks = cols // 32
    r = min(rows, CHECK_ROWS)
    rng = np.random.default_rng(rows + 3 * cols + 7 * n)
    if vision:
        hq, hs = oracle.quantize_q8(orc.vision_weights_f32(rng, r, cols), r, cols)
    else:
        hq, hs = orc.q4_weights(rng, r, cols) if q4 else orc.q8_weights(rng, r, cols)
    xs = orc.activations(rng, n, cols)
    gen = torch.Generator(device="cuda")
    gen.manual_seed(1)
    qs, sc = device_weights(torch, L, fmt, rows, cols, gen)
    qs.view(torch.uint8)[:hq.nbytes] = torch.from_numpy(hq.view(np.uint8)).cuda()
    sc.view(torch.uint8)[:hs.nbytes] = torch.from_numpy(hs.view(np.uint8)).cuda()
    x = torch.from_numpy(xs).cuda()
    xq = torch.zeros(n * cols, dtype=torch.int8, device="cuda")
    xsc = torch.zeros(n * blocks + 4, device="cuda")
    ys = torch.full((n * rows,), float("nan"), device="cuda")
    path = L.dn_linear_path(1 if q4 else 0, qs.data_ptr(), sc.data_ptr(), x.data_ptr(), xq.data_ptr(),
                            rows, cols, n, 1)
    rc = L.dn_linear(1 if q4 else 0, qs.data_ptr(), sc.data_ptr(), x.data_ptr(), xq.data_ptr(),
                     xsc.data_ptr(), ys.data_ptr(), rows, cols, n, rows, 1, -1, 0,
                     torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    if rc != 0 or L.dn_device_status(1) != 0:
        return path, False, None
    got = ys.view(n, rows)[:, :r].contiguous().cpu().numpy().reshape(-1)
    if path == 1:
        ref, mag = oracle.reference_f64(fmt, hq, hs, xs, r, cols, n, 1)
        err = orc.max_rel_err(got, ref, mag)
        return path, bool(err < 1e-5), err
    want, _, _ = oracle.gemm(fmt, hq, hs, xs, r, cols, n, 1)
    return path, bool(np.array_equal(got.view(np.uint32), want.view(np.uint32))), 0.0


def cpu_linear_us(ref, fmt, rows, cols, n, threads, budget_s=2.0):
    """us per call of the reference's lab_gemm_q4 / _q8 (mode 1) on this host."""
    from oracle import oracle as orc
    rng = np.random.default_rng(rows + cols + n)
    qs, sc = orc.q4_weights(rng, rows, cols) if fmt == "q4" else orc.q8_weights(rng, rows, cols)
    xs = orc.activations(rng, n, cols)
    out = (np.zeros(n * rows, np.float32), np.zeros(n * cols, np.int8),
           np.zeros(n * (cols // 32) + 1, np.float32))
    ref.gemm(fmt, qs, sc, xs, rows, cols, n, 1, threads, out)
    times, t_end = [], time.perf_counter() + budget_s
    while len(times) < 3 or (time.perf_counter() < t_end and len(times) < 50):
        t0 = time.perf_counter()
        ref.gemm(fmt, qs, sc, xs, rows, cols, n, 1, threads, out)
        times.append(time.perf_counter() - t0)
    return statistics.median(times) * 1e6


# The configuration cases the default bench line carries ("configs" key):
# (config, case, fmt, rows, cols, n, vision weights).
COMPACT_CASES = [("c1", "mlp_up_q4_gemv", "q4", 6144, 2048, 1, False),
                 ("c2", "gate_q8_gemv", "q8", 6144, 2048, 1, False),
                 ("c4", "gate_up_q4_m512", "q4", 6144, 2048, 512, False),
                 ("c5", "qkv_q8_m1024", "q8", 3456, 1152, 1024, True),
                 ("c5", "lm_head_q8_m16", "q8", VOCAB, HIDDEN, 16, False)]


# Products straight on GGUF blocks (dn_gguf_linear_qa, no split), one token.
GGUF_CASES = [("c1", "mlp_up_q4_gguf", "q4", 6144, 2048),
              ("c5", "lm_head_q8_gguf", "q8", VOCAB, HIDDEN)]


def gguf_device_blocks(torch, fmt, rows, cols, gen):
    """A matrix as a GGUF file stores it, on the device: per 32-block an fp16
    scale (Q4_0 U[0.002, 0.02], Q8_0 U[0.001, 0.01], the configs' ranges) and
    the 16 nibble bytes / 32 int8 (U[-127, 127])."""
    nb = rows * (cols // 32)
    size = 18 if fmt == "q4" else 34
    raw = torch.empty((nb, size), dtype=torch.uint8, device="cuda")
    if fmt == "q4":
        raw[:, 2:] = torch.randint(0, 256, (nb, 16), dtype=torch.uint8, device="cuda", generator=gen)
        lo, hi = 0.002, 0.02
    else:
        raw[:, 2:] = torch.randint(-127, 128, (nb, 32), dtype=torch.int8, device="cuda",
                                   generator=gen).view(torch.uint8)
        lo, hi = 0.001, 0.01
    sc = torch.empty(nb, device="cuda").uniform_(lo, hi, generator=gen).half()
    raw[:, :2] = sc.view(torch.uint8).view(nb, 2)
    return raw


def time_gguf(torch, L, oracle, fmt, rows, cols, steps, warmup):
    """us per one-token product on GGUF blocks (the activation quantize to QA
    blocks included, as in time_linear), blocks rotating through copies past
    twice the L2; and its first CHECK_ROWS rows against the oracle on the
    blocks split as the reference's loader splits them."""
    q4 = fmt == "q4"
    per_copy = rows * (cols // 32) * (18 if q4 else 34)
    l2 = torch.cuda.get_device_properties(0).L2_cache_size
    copies = max(1, -(-2 * l2 // per_copy))
    gen = torch.Generator(device="cuda")
    gen.manual_seed(rows * 13 + cols)
    raw0 = gguf_device_blocks(torch, fmt, rows, cols, gen)
    sets = [raw0] + [raw0.clone() for _ in range(copies - 1)]
    x = torch.randn(cols, device="cuda", generator=gen)
    xa = torch.zeros(cols // 32 * 36, dtype=torch.uint8, device="cuda")
    ys = torch.full((rows,), float("nan"), device="cuda")
    stream = torch.cuda.Stream()

    def launch(i, h):
        rc = L.dn_quantize_qa(x.data_ptr(), xa.data_ptr(), 1, cols, cols // 32 * 36, h)
        if rc == 0:
            rc = L.dn_gguf_linear_qa(1 if q4 else 0, sets[i % copies].data_ptr(), xa.data_ptr(), ys.data_ptr(),
                                     rows, cols, 1, h)
        if rc != 0:
            raise RuntimeError(L.dn_error_string(rc).decode())

    with torch.cuda.stream(stream):
        for i in range(warmup):
            launch(i, stream.cuda_stream)
        torch.cuda.synchronize()
        r = min(rows, CHECK_ROWS)
        raw = raw0[:r * (cols // 32)].cpu().numpy()
        if q4:
            qs, sc = raw[:, 2:].ravel().copy(), raw[:, :2].ravel().copy().view(np.uint16)
        else:
            qs, sc = raw[:, 2:].ravel().copy(), raw[:, :2].copy().view(np.float16).astype(np.float32).ravel()
        want, _, _ = oracle.gemm(fmt, qs, sc, x.cpu().numpy(), r, cols, 1, 1)
        launch(0, stream.cuda_stream)
        torch.cuda.synchronize()
        ok = bool(np.array_equal(ys[:r].cpu().numpy().view(np.uint32), want.view(np.uint32)))
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            for i in range(steps):
                launch(i, torch.cuda.current_stream().cuda_stream)
        graph.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        graph.replay()
        e1.record(stream)
        torch.cuda.synchronize()
    del graph
    if L.dn_device_status(1) != 0:
        raise SystemExit("kernel bounded wait timed out")
    return e0.elapsed_time(e1) * 1e3 / steps, ok, copies


def run_configs_compact(args, torch, L):
    """Configs 1, 2, 4, 5 and the lm_head sweep in short: per case the GPU time
    per dn_linear launch (graph-replayed, operands past L2) as HBM GB/s and
    int8 TOPS against the measured peaks, the reference's CPU kernels on the
    same case (oracle/_ref, all host threads) and a check of the GPU's output
    against the oracle outside the timed region."""
    from oracle import oracle as orc
    bind_cpu_threads()
    peaks = {}
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            peaks = json.load(f)
    except OSError:
        pass
    hbm = float(peaks.get("hbm_gbs", 6650.0))
    int8 = 2.0 * float(peaks.get("bf16_tflops", 1590.0))
    try:
        ref = orc.Reference()
    except FileNotFoundError:
        ref = None
    oracle = orc.Oracle()
    threads = host_threads()
    out = []
    for cfg, name, fmt, rows, cols, n, vision in COMPACT_CASES:
        path, ok, err = check_linear(torch, L, oracle, fmt, rows, cols, n, vision)
        us, _, copies = time_linear(torch, L, fmt, rows, cols, n, args.config_steps, 3, vision)
        alg_bytes = rows * cols // 32 * (18 if fmt == "q4" else 34) + 4 * n * (cols + rows)
        ops = 2.0 * n * rows * cols
        res = {"config": cfg, "case": name, "fmt": fmt, "rows": rows, "cols": cols, "n": n,
               "path": {0: "gemv", 1: "tcgen05", 2: "generic"}.get(path, path), "us": us,
               "gbs_algorithmic": alg_bytes / us / 1e3, "hbm_frac": alg_bytes / us / 1e3 / hbm,
               "tops": ops / us / 1e6, "int8_frac": ops / us / 1e6 / int8,
               "check": ("bit-exact with the oracle" if path != 1 else
                         "max relative error vs the oracle's double reference (bound 1e-5)"),
               "check_rows": min(rows, CHECK_ROWS), "check_ok": ok, "max_rel_err": err,
               "weights": "bf16 N(0,0.02) -> lab_quantize_q8" if vision else "config distribution",
               "copies": copies}
        if ref is not None:
            cus = cpu_linear_us(ref, fmt, rows, cols, n, threads, budget_s=1.0)
            res.update(cpu_reference_us=cus, cpu_threads=threads, gpu_speedup=cus / us)
        out.append(res)
    for cfg, name, fmt, rows, cols in GGUF_CASES:
        us, ok, copies = time_gguf(torch, L, oracle, fmt, rows, cols, args.config_steps, 3)
        alg_bytes = rows * cols // 32 * (18 if fmt == "q4" else 34) + 4 * (cols + rows)
        res = {"config": cfg, "case": name, "fmt": fmt, "rows": rows, "cols": cols, "n": 1,
               "path": "gguf gemv (the file's interleaved blocks, no split)", "us": us,
               "gbs_algorithmic": alg_bytes / us / 1e3, "hbm_frac": alg_bytes / us / 1e3 / hbm,
               "check": "bit-exact with the oracle on the blocks split as the reference's loader splits them",
               "check_rows": min(rows, CHECK_ROWS), "check_ok": ok, "copies": copies}
        if ref is not None:
            cus = cpu_linear_us(ref, fmt, rows, cols, 1, threads, budget_s=1.0)
            res.update(cpu_reference_us=cus, cpu_threads=threads, gpu_speedup=cus / us)
        out.append(res)
    return {"cases": out, "peaks": {"hbm_gbs": hbm, "int8_tops": int8,
                                    "int8_source": "2 x MEASURED_PEAKS.json bf16_tflops"},
            "timing": f"{args.config_steps} graph-replayed launches per case, operands rotating past "
                      "2 x L2, CUDA events; activation quantize included"}


def run_drain_workload(args):
    """The tensor-core GEMM's own ceiling: dn_drain_probe runs only its
    per-block drain (TMEM load, exact conversion, rank-1 scale product,
    f32x2 accumulate) on one CTA per SM. Reports output element-blocks drained
    per clock per SM (SM clock sampled during the run) and the int8 TOPS that
    rate allows a GEMM (64 ops per element-block), beside the int8 peak."""
    import torch
    from dianoia_b200 import _lib
    L = _lib.lib()
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    nst = max(args.steps, 1) * 10
    out = torch.empty(sms * 576, dtype=torch.float32, device="cuda")
    stream = torch.cuda.Stream()
    for _ in range(max(args.warmup, 3)):
        _lib.check(L.dn_drain_probe(sms, nst, out.data_ptr(), stream.cuda_stream), "dn_drain_probe")
    torch.cuda.synchronize()
    times = []
    with ClockSampler(0) as clocks:
        for _ in range(5):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            _lib.check(L.dn_drain_probe(sms, nst, out.data_ptr(), stream.cuda_stream), "dn_drain_probe")
            e1.record(stream)
            torch.cuda.synchronize()
            times.append(e0.elapsed_time(e1) * 1e-3)
    t = min(times)
    ck = clocks.summary() or {}
    mhz = float(ck.get("sm_mhz") or 1965.0)
    eb = sms * 128 * 64 * 4 * nst
    peaks = {}
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            peaks = json.load(f)
    except OSError:
        pass
    int8 = 2.0 * float(peaks.get("bf16_tflops", 1590.0))
    res = {"metric": "tcgen05 GEMM drain ceiling", "sms": sms, "stages": nst, "seconds": t,
           "element_blocks_per_clk_per_sm": eb / (t * mhz * 1e6 * sms), "sm_mhz": mhz,
           "ceiling_tops": eb * 64 / t / 1e12, "int8_peak_tops": int8,
           "ceiling_frac_of_int8_peak": eb * 64 / t / 1e12 / int8, "clocks": ck,
           "what": "per block: tcgen05.ld 32x32b.x32, exact int->float (f32x2 add), rank-1 scale "
                   "product (f32x2 mul), f32x2 fma; 16 drain warps per SM, no MMA, copy or barrier"}
    print(json.dumps(res), flush=True)


# Config 5 and the lm_head M sweep at N GPUs (row-sharded weights, the
# output blocks all-gathered): (case, fmt, rows, cols, n, vision weights).
SHARDED_CASES = ([(f"vision_{nm}_m1024", "q8", r, c, 1024, True)
                  for nm, r, c in [("qkv", 3456, 1152), ("o", 1152, 1152), ("fc1", 4304, 1152),
                                   ("fc2", 1152, 4320)]]
                 + [(f"lm_head_m{m}", "q8", VOCAB, HIDDEN, m, False) for m in (1, 2, 4, 8, 16, 32, 64)])


class FusedRegion:
    """`nbytes` of device memory on every rank that every other rank maps
    (dn_peer_alloc / dn_peer_open, handles exchanged with the process group);
    bases[p] is rank p's region as mapped here."""

    def __init__(self, L, dist, rank, world, nbytes):
        from dianoia_b200 import _lib
        self.L, self.dist, self.world = L, dist, world
        nbytes = (nbytes + 4095) // 4096 * 4096
        base = ctypes.c_void_p()
        handle = (ctypes.c_uint8 * _lib.DN_PEER_HANDLE_BYTES)()
        _lib.check(L.dn_peer_alloc(nbytes, ctypes.byref(base), handle), "dn_peer_alloc")
        self.base = base.value
        handles = [bytes(handle)]
        if world > 1:
            handles = [None] * world
            dist.all_gather_object(handles, bytes(handle))
        self.bases, self.opened = [], []
        for p in range(world):
            if p == rank:
                self.bases.append(self.base)
                continue
            ptr = ctypes.c_void_p()
            h = (ctypes.c_uint8 * _lib.DN_PEER_HANDLE_BYTES).from_buffer_copy(handles[p])
            _lib.check(L.dn_peer_open(h, ctypes.byref(ptr)), "dn_peer_open")
            self.bases.append(ptr.value)
            self.opened.append(ptr.value)
        if world > 1:
            dist.barrier()  # every region mapped everywhere before any rank stores into it

    def close(self):
        if self.world > 1:
            self.dist.barrier()  # no rank still stores into another's region
        for p in self.opened:
            self.L.dn_peer_close(p)
        self.opened = []
        if self.world > 1:
            self.dist.barrier()
        if self.base:
            self.L.dn_peer_free(self.base)
            self.base = None


def run_configs_sharded(args, rank, world, local_rank):
    """Configs 5 and the lm_head sweep on N GPUs: each rank holds its row
    slice of the weights (rows * p // N ..) and computes its column block of
    Y[n, rows] for the whole batch of tokens. By default the gather is fused
    into the product: every rank's kernel stores its block into every rank's
    Y over NVLink and counts it on the peers' counters (dn_linear_allgather,
    or dn_linear_qa_allgather for one token), and each rank's step ends in a
    bounded wait for all the blocks; the steps replay from a CUDA graph.
    With --gather nccl, dn_linear on the slice is followed by an NCCL
    all-gather of the column blocks (padded to the widest slice, then laid
    out token-major by one copy). Everything is inside the timed region;
    time is the max over ranks. One JSON line per case from rank 0."""
    import torch
    import torch.distributed as dist
    from datetime import timedelta
    from dianoia_b200 import _lib
    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=device)
    L = _lib.lib()
    peaks = {}
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            peaks = json.load(f)
    except OSError:
        pass
    int8 = 2.0 * float(peaks.get("bf16_tflops", 1590.0))
    hbm = float(peaks.get("hbm_gbs", 6650.0))
    stream = torch.cuda.Stream(device=device)
    for name, fmt, rows, cols, n, vision in SHARDED_CASES:
        if args.cases and not re.search(args.cases, name):
            continue
        r0, r1 = row_split(rows, rank, world, False)
        rr = r1 - r0
        width = max(row_split(rows, p, world, False)[1] - row_split(rows, p, world, False)[0]
                    for p in range(world))
        blocks = cols // 32
        gen = torch.Generator(device=device)
        gen.manual_seed(1000 + rank)
        qs, sc = device_weights(torch, L, fmt, rr, cols, gen, vision)
        xs = torch.randn(n * cols, device=device, generator=torch.Generator(device=device).manual_seed(7))
        xq = torch.zeros(n * cols, dtype=torch.int8, device=device)
        xsc = torch.zeros(n * blocks + 4, device=device)
        spans = [row_split(rows, p, world, False) for p in range(world)]
        # The fused gathers: one token on the GEMV (dn_linear_qa_allgather,
        # its count one per 32-row tile), more on the tensor-core GEMM
        # (dn_linear_allgather, one count per rank).
        fused = args.gather == "fused"
        if fused:
            # Every rank's Y[n, rows] (then its counter and wait word) in peer
            # memory; each rank's GEMM epilogue stores its column block into
            # every copy over NVLink (dn_linear_allgather), then a bounded
            # wait on this rank's counter for all ranks' tiles.
            region = FusedRegion(L, dist, rank, world, 4 * n * rows + 256)
            ys_arr = (ctypes.c_void_p * world)(*region.bases)
            cnt_arr = (ctypes.c_void_p * world)(*[b + 4 * n * rows for b in region.bases])
            counter = region.bases[rank] + 4 * n * rows
            expect = counter + 4
            tiles = world if n > 1 else sum(-(-(b - a) // 32) for a, b in spans)
            xa = torch.zeros(blocks * 36, dtype=torch.uint8, device=device) if n == 1 else None
        else:
            ys = torch.zeros(n * width, device=device)  # [n, width]: this rank's block, padded
            gathered = torch.empty(world * n * width, device=device)
            full = torch.empty(n * rows, device=device)

        def step():
            if fused and n == 1:
                rc = L.dn_quantize_qa(xs.data_ptr(), xa.data_ptr(), 1, cols, blocks * 36, stream.cuda_stream)
                if rc == 0:
                    rc = L.dn_linear_qa_allgather(1 if fmt == "q4" else 0, qs.data_ptr(), sc.data_ptr(),
                                                  xa.data_ptr(), rr, cols, r0, ys_arr, cnt_arr, world, 1,
                                                  stream.cuda_stream)
                if rc == 0:
                    rc = L.dn_peer_wait(counter, expect, tiles, stream.cuda_stream)
                if rc != 0:
                    raise RuntimeError(L.dn_error_string(rc).decode())
                return
            if fused:
                rc = L.dn_linear_allgather(1 if fmt == "q4" else 0, qs.data_ptr(), sc.data_ptr(), xs.data_ptr(),
                                           xq.data_ptr(), xsc.data_ptr(), rr, cols, n, r0, rows, ys_arr, cnt_arr,
                                           world, stream.cuda_stream)
                if rc == 0:
                    rc = L.dn_peer_wait(counter, expect, tiles, stream.cuda_stream)
                if rc != 0:
                    raise RuntimeError(L.dn_error_string(rc).decode())
                return
            rc = L.dn_linear(1 if fmt == "q4" else 0, qs.data_ptr(), sc.data_ptr(), xs.data_ptr(),
                             xq.data_ptr(), xsc.data_ptr(), ys.data_ptr(), rr, cols, n, width, 1, -1, 0,
                             stream.cuda_stream)
            if rc != 0:
                raise RuntimeError(L.dn_error_string(rc).decode())
            if world > 1:
                dist.all_gather_into_tensor(gathered, ys)
                g = gathered.view(world, n, width)
                fv = full.view(n, rows)
                for p, (a, b) in enumerate(spans):
                    fv[:, a:b].copy_(g[p, :, :b - a])

        with torch.cuda.stream(stream):
            for _ in range(3):
                step()
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        steps = max(args.steps, 1)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        graph = None
        if fused:
            # The fused steps replay from a CUDA graph (no collective inside:
            # the ranks meet in the bounded counter waits).
            with torch.cuda.stream(stream):
                graph = torch.cuda.CUDAGraph()
                with torch.cuda.graph(graph, stream=stream):
                    for _ in range(steps):
                        step()
                graph.replay()
            torch.cuda.synchronize()
            if world > 1:
                dist.barrier()
            torch.cuda.synchronize()
        with torch.cuda.stream(stream):
            e0.record(stream)
            if graph is not None:
                graph.replay()
            else:
                for _ in range(steps):
                    step()
            e1.record(stream)
        torch.cuda.synchronize()
        del graph
        t = torch.tensor([e0.elapsed_time(e1) * 1e3 / steps], dtype=torch.float64, device=device)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        us = float(t.item())
        ops = 2.0 * n * rows * cols
        wbytes = rows * blocks * 34
        check = None
        if fused:
            # Outside the timed region: every rank's copy of Y is the same,
            # and this rank's own columns equal dn_linear on its slice.
            torch.cuda.synchronize()
            mine = torch.as_tensor(_DevArray(region.bases[rank], n * rows), device=device).view(n, rows)
            own = torch.empty(n * rr, device=device)
            rc = L.dn_linear(1 if fmt == "q4" else 0, qs.data_ptr(), sc.data_ptr(), xs.data_ptr(), xq.data_ptr(),
                             xsc.data_ptr(), own.data_ptr(), rr, cols, n, rr, 1, -1, 0, stream.cuda_stream)
            torch.cuda.synchronize()
            got = mine[:, r0:r1].contiguous()
            same_path = n == 1 or L.dn_linear_path(1 if fmt == "q4" else 0, qs.data_ptr(), sc.data_ptr(),
                                                   xs.data_ptr(), xq.data_ptr(), rr, cols, n, 1) == 1
            if same_path:  # the same kernel: value for value
                own_ok = rc == 0 and bool(torch.equal(got.view(torch.int32), own.view(n, rr).view(torch.int32)))
            else:  # dn_linear picks the GEMV for these few tokens: the tensor-core bound
                ref = own.view(n, rr).double()
                own_ok = rc == 0 and bool(((got.double() - ref).abs().max() <=
                                           1e-5 * ref.abs().max().clamp_min(1e-30)).item())
            sums = torch.tensor([float(mine.double().sum().item())], dtype=torch.float64, device=device)
            allsums = [torch.zeros_like(sums) for _ in range(world)]
            if world > 1:
                dist.all_gather(allsums, sums)
            else:
                allsums = [sums]
            flags = torch.tensor([1 if own_ok else 0], device=device)
            if world > 1:
                dist.all_reduce(flags, op=dist.ReduceOp.MIN)
            check = {"copies_identical": len({float(x.item()) for x in allsums}) == 1,
                     "own_columns_match_dn_linear_on_all_ranks": bool(flags.item() == 1),
                     "match": "bit for bit where dn_linear takes the same kernel, else within 1e-5 of the "
                              "slice's largest output"}
        if rank == 0:
            print(json.dumps({"case": name, "n_gpus": world, "fmt": fmt, "rows": rows, "cols": cols, "n": n,
                              "rows_per_gpu": width, "us": us, "tops": ops / us / 1e6,
                              "int8_frac_per_gpu": ops / us / 1e6 / (int8 * world),
                              "weight_gbs": wbytes / us / 1e3,
                              "hbm_frac_per_gpu": wbytes / us / 1e3 / (hbm * world),
                              "includes": ("dn_quantize_qa + dn_linear_qa_allgather on each rank's row "
                                           "slice (the GEMV's outputs stored into every rank's copy over "
                                           "NVLink) + dn_peer_wait" if fused and n == 1 else
                                           "dn_linear_allgather on each rank's row slice (activation "
                                           "quantize included; the output columns stored into every rank's "
                                           "Y over NVLink inside the tensor-core GEMM's epilogue) + "
                                           "dn_peer_wait" if fused else
                                           "dn_linear on each rank's row slice (activation quantize "
                                           "included) + NCCL all-gather of the output blocks + "
                                           "token-major layout copy" if world > 1 else "dn_linear"),
                              "check": check,
                              "weights": "bf16 N(0,0.02) -> lab_quantize_q8" if vision else "config distribution",
                              "timing": f"{steps} steps" + (" replayed from a CUDA graph" if fused else
                                                            " launched eagerly") +
                                        ", CUDA events, max over ranks; operands L2-resident between "
                                        "launches (one copy per rank)"}), flush=True)
        torch.cuda.synchronize()
        if fused:
            region.close()
        else:
            del ys, gathered, full
        del qs, sc, xs, xq, xsc
        torch.cuda.empty_cache()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def run_configs_workload(args):
    """One JSON line per BASELINE config case: the GPU time per dn_linear
    launch (graph-replayed, operands past L2) as HBM GB/s for the decode
    GEMVs and int8 TOPS for the GEMMs, each against its measured peak, and the
    reference's CPU kernels (oracle/_ref, all host threads) on the same case."""
    import torch
    from dianoia_b200 import _lib
    L = _lib.lib()
    peaks = {}
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            peaks = json.load(f)
    except OSError:
        pass
    hbm = float(peaks.get("hbm_gbs", 6650.0))
    int8 = 2.0 * float(peaks.get("bf16_tflops", 1590.0))
    ref = None
    if args.cpu_tokens > 0:
        from oracle import oracle as orc
        bind_cpu_threads()
        try:
            ref = orc.Reference()
        except FileNotFoundError:
            ref = None
    threads = host_threads()
    for cfg, name, fmt, rows, cols, n in CONFIG_CASES:
        vision = cfg == "c5" and not name.startswith("lm_head")
        us, path, copies = time_linear(torch, L, fmt, rows, cols, n, args.steps, max(args.warmup, 3), vision)
        blocks = rows * cols // 32
        alg_bytes = blocks * (18 if fmt == "q4" else 34) + 4 * n * (cols + rows)
        ops = 2.0 * n * rows * cols
        res = {"config": cfg, "case": name, "fmt": fmt, "rows": rows, "cols": cols, "n": n,
               "path": path, "us": us, "gbs_algorithmic": alg_bytes / us / 1e3,
               "hbm_frac": alg_bytes / us / 1e3 / hbm, "tops": ops / us / 1e6,
               "int8_frac": ops / us / 1e6 / int8, "copies": copies}
        if ref is not None:
            cus = cpu_linear_us(ref, fmt, rows, cols, n, threads)
            res["cpu_reference_us"] = cus
            res["cpu_threads"] = threads
            res["gpu_speedup"] = cus / us
        print(json.dumps(res), flush=True)


def run_e2e_device_api(args, torch, stack, step, stream, logits_dev, world, device, full_logits):
    """Token loop through this library's device C-ABI with host buffers: per
    token x0 is copied in from pinned host memory, the token's launches run
    (the captured graph of dn_quantize_qa, dn_linear_qa and, on N > 1 GPUs,
    dn_linear_qa_allgather + dn_peer_wait), and the whole logits are copied
    back to pinned host memory and synchronized. Host wall clock per token,
    max over ranks."""
    steps = args.e2e_steps
    if steps <= 0:
        return None
    x0_h = stack.x0.cpu().pin_memory()
    logits_h = torch.empty(VOCAB, dtype=torch.float32).pin_memory()

    def one_token():
        with torch.cuda.stream(stream):
            stack.x0.copy_(x0_h, non_blocking=True)
            step()
            logits_h.copy_(logits_dev, non_blocking=True)
        stream.synchronize()

    for _ in range(3):
        one_token()
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
    t0 = time.perf_counter()
    for _ in range(steps):
        one_token()
    dt = time.perf_counter() - t0
    t = torch.tensor([dt], dtype=torch.float64, device=device)
    if world > 1:
        import torch.distributed as dist
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    dt = float(t.item())
    same = bool(np.array_equal(logits_h.numpy().view(np.uint32), full_logits.cpu().numpy().view(np.uint32)))
    return {"value": steps / dt, "unit": "tokens/s", "h2d_bytes_per_step": 4 * HIDDEN,
            "d2h_bytes_per_step": 4 * VOCAB,
            "api": "the library's device C-ABI with host buffers: per token x0 copied in from pinned "
                   "memory, the token's launches (dn_quantize_qa, dn_linear_qa" +
                   (", dn_linear_qa_allgather, dn_peer_wait" if world > 1 else "") +
                   ", one CUDA graph), the whole logits copied back and synchronized",
            "steps": steps, "timing": "host wall clock, max over ranks",
            "logits_match_device_run": same}


def run_e2e(args, stack, L, torch, rank, world, gather, device, full_logits):
    """Token loop through lab_gemm_q8 with host activations / outputs."""
    steps = args.e2e_steps
    if steps <= 0:
        return None
    maxc = max(m["cols"] for m in stack.mats)
    xq = np.zeros(maxc, np.int8)
    xsc = np.zeros(maxc // 32 + 1, np.float32)
    host = {n: np.zeros(b.numel(), np.float32) for n, b in stack.bufs.items()}
    x0 = stack.x0.cpu().numpy()
    dev_tmp = {n: b.clone() for n, b in stack.bufs.items()} if world > 1 else None
    h2d = d2h = 0

    def one_token():
        nonlocal h2d, d2h
        h2d = d2h = 0
        for m in stack.mats:
            name = m["name"]
            src = INPUT_OF[name]
            xin = x0 if src is None else np.ascontiguousarray(host[src][:m["cols"]])
            out = host[name]
            rl = m["r1"] - m["r0"]
            ys = out[m["r0"]:m["r1"]]
            L.lab_gemm_q8(m["qs"].data_ptr(), m["scales"].data_ptr(), xin.ctypes.data,
                          xq.ctypes.data, xsc.ctypes.data, ys.ctypes.data, rl, m["cols"], 1, 1, 1)
            h2d += xin.nbytes
            d2h += ys.nbytes + m["cols"] + m["cols"] // 32 * 4
            if world > 1 and rl < m["rows"]:
                # All-gather of the row slices (any split): each rank adds
                # its rows into zeros, exactly.
                d = dev_tmp[name]
                d.zero_()
                d[m["r0"]:m["r1"]].copy_(torch.from_numpy(ys))
                import torch.distributed as dist
                dist.all_reduce(d)
                out[:] = d.cpu().numpy()
        if L.dn_last_error() != 0:
            raise RuntimeError("lab_gemm_q8 failed")

    for _ in range(2):
        one_token()
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
    t0 = time.perf_counter()
    for _ in range(steps):
        one_token()
    dt = time.perf_counter() - t0
    t = torch.tensor([dt], dtype=torch.float64, device=device)
    if world > 1:
        import torch.distributed as dist
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    dt = float(t.item())
    # Same logits as the device-resident run.
    same = bool(np.array_equal(host["lm_head"].view(np.uint32),
                               full_logits.cpu().numpy().view(np.uint32)))
    return {"value": steps / dt, "unit": "tokens/s", "h2d_bytes_per_step": h2d,
            "d2h_bytes_per_step": d2h, "api": "lab_gemm_q8 (host x / y, device weights)",
            "steps": steps, "logits_match_device_run": same}


def run_e2e_gpu_layer(args, stack, L, torch):
    """Token loop through dianoia's GPU-layer C-ABI (lab_gpu_*), the way its
    GpuForward drives a GPU: weights in GPU buffers (uploaded once), and per
    token the host writes x0 into a host-visible buffer, records all 113
    products into one command buffer (each projection's output feeding the
    next inside an activation buffer), commits with wait and reads the
    logits. The commit copies x0 in and every product's outputs back; those
    copies and the host's encode calls are inside the timed region."""
    steps = args.e2e_steps
    if steps <= 0 or L.lab_gpu_init() != 1:
        return None
    handles = []
    try:
        mats = wrap_stack(L, stack, handles)
        # Activation buffer: x0, then one output region per projection kind.
        offs, at = {"x0": 0}, HIDDEN
        for name in ("qkv", "o", "gate_up", "down"):
            offs[name] = at
            at += OUT_ROWS[name]
        act = L.lab_gpu_buffer(4 * at)
        logits_h = L.lab_gpu_readback_buffer(4 * VOCAB)
        handles += [act, logits_h]
        act_view = np.ctypeslib.as_array((ctypes.c_float * at).from_address(L.lab_gpu_contents(act)))
        logits_view = np.ctypeslib.as_array(
            (ctypes.c_float * VOCAB).from_address(L.lab_gpu_contents(logits_h)))
        x0 = stack.x0.cpu().numpy()
        logits = np.zeros(VOCAB, np.float32)

        # One row per product, as lab_gpu_enc_matmul_q8 takes them.
        table = []
        for m, (h, sc_at) in zip(stack.mats, mats):
            name = m["name"]
            src = INPUT_OF[name]
            x_off = 4 * offs["x0" if src is None else src]
            y, y_off = (logits_h, 0) if name == "lm_head" else (act, 4 * offs[name])
            table.append([0, h, 0, sc_at, act, x_off, y, y_off, m["rows"], m["cols"], 1])
        table = np.ascontiguousarray(np.array(table, np.int64))

        def one_token(batch):
            act_view[:HIDDEN] = x0
            L.lab_gpu_begin()
            if batch:
                L.dn_gpu_enc_batch(table.ctypes.data, len(table))
            else:
                for r in table.tolist():
                    L.lab_gpu_enc_matmul_q8(*r[1:])
            if L.lab_gpu_commit(1) != 1:
                raise RuntimeError("lab_gpu_commit failed")
            # The logits are read in place in the pinned mirror (the commit's
            # device-to-host copy put them there), as a Dart caller reads them.
            dev_ms.append(L.lab_gpu_last_ms())

        dev_ms = []

        def timed(batch):
            for _ in range(3):
                one_token(batch)
            dev_ms.clear()
            t0 = time.perf_counter()
            for _ in range(steps):
                one_token(batch)
            return steps / (time.perf_counter() - t0)

        per_call = timed(False)
        value = timed(True)
        commit_ms = float(np.median(dev_ms))
        logits[:] = logits_view
        same = bool(np.array_equal(logits.view(np.uint32),
                                   stack.bufs["lm_head"].cpu().numpy().view(np.uint32)))
        d2h = 4 * (at - HIDDEN) + 4 * VOCAB
        return {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 4 * HIDDEN,
                "d2h_bytes_per_step": d2h,
                "api": "lab_gpu_* (dianoia's GPU-layer ABI: host-visible buffers; per token "
                       "lab_gpu_begin, the 113 products recorded by one dn_gpu_enc_batch call, "
                       "lab_gpu_commit(wait=1))",
                "commit_device_ms": commit_ms,
                "commit_device_note": "median GPU time of one commit's graph (uploads, 113 "
                                      "products, downloads), from lab_gpu_last_ms",
                "per_call_encode_tokens_s": per_call,
                "per_call_encode_note": "the same loop recording each product with its own "
                                        "lab_gpu_enc_matmul_q8 call: a Python ctypes call costs "
                                        "~3 us, a Dart @Native leaf call tens of ns",
                "steps": steps, "logits_match_device_run": same}
    finally:
        for h in handles:
            L.lab_gpu_release(h)


def wrap_stack(L, stack, handles):
    """Each matrix of the stack as one GPU-layer buffer: values, then the
    scales at the next 64-byte boundary; returns (handle, scales offset)."""
    mats = []
    for m in stack.mats:
        qs = m["qs"].cpu().numpy().view(np.uint8)
        sc = m["scales"].cpu().numpy().view(np.uint8)
        at = (qs.size + 63) // 64 * 64
        raw = np.zeros(at + sc.size, np.uint8)
        raw[:qs.size] = qs
        raw[at:] = sc
        h = L.lab_gpu_wrap(raw.ctypes.data, raw.size)
        if h < 0:
            raise RuntimeError("lab_gpu_wrap failed")
        handles.append(h)
        mats.append((h, at))
    return mats


def run_neighbours(args, stack, L, context=0):
    """The decode stack with the neighbours of its products, through the GPU
    layer as dianoia's GpuForward encodes a Qwen3 layer (gpu.dart:1100-1190)
    less the attention (out of this path: o reads q's rows in its place):
    norm, qkv, o, residual add, norm, gate, up, SwiGLU, down, residual add;
    then the final norm and the lm_head. The same weights as the projection
    stack (gate and up are the two row halves of gate_up), RMSNorm weights
    1 + 0.1 N(0, 1), eps 1e-6. Timed per token like `e2e` (host writes x0,
    one dn_gpu_enc_batch, lab_gpu_commit(wait=1)), fused (norms hand QA
    blocks to their products, SwiGLU and the adds run in product epilogues)
    and with every op its own kernel on f32 inputs (dn_gpu_set_fusion(0), the
    reference layer's dispatch structure).

    With `context` > 0 the attention is there too, as GpuForward records it
    (gpu.dart:1100-1180): q and k per-head RMSNorm + RoPE in place, the
    token's k and v copied into device-resident KV caches (dn_gpu_device_buffer)
    at row `context`, causal attention over the `context` + 1 cached rows, and
    o reading the attention's output: a whole Qwen3-1.7B-shaped decode step."""
    steps = args.neighbour_steps
    if steps <= 0 or L.lab_gpu_init() != 1:
        return None
    handles = []
    try:
        mats = wrap_stack(L, stack, handles)
        rng = np.random.default_rng(7)
        norms = (1 + 0.1 * rng.standard_normal((2 * LAYERS + 1) * HIDDEN)).astype(np.float32)
        small = L.lab_gpu_wrap(norms.ctypes.data, norms.nbytes)
        handles.append(small)
        sizes = {"x": HIDDEN, "a": HIDDEN, "qkv": OUT_ROWS["qkv"], "m": HIDDEN, "g": INTER,
                 "u": INTER, "attn": HEADS * HEAD_DIM, "rope": 2 * HEAD_DIM, "q": HEADS * HEAD_DIM}
        kv_dim = KV_HEADS * HEAD_DIM
        caches = []
        if context > 0:
            qk = (1 + 0.1 * rng.standard_normal(LAYERS * 2 * HEAD_DIM)).astype(np.float32)
            qk_norms = L.lab_gpu_wrap(qk.ctypes.data, qk.nbytes)
            handles.append(qk_norms)
            init = rng.standard_normal((context + 1) * kv_dim).astype(np.float32)
            stage = L.lab_gpu_buffer(init.nbytes)
            handles.append(stage)
            np.ctypeslib.as_array((ctypes.c_float * init.size).from_address(L.lab_gpu_contents(stage)))[:] = init
            L.lab_gpu_begin()
            for _ in range(2 * LAYERS):  # random history in every layer's keys and values
                c = L.dn_gpu_device_buffer(init.nbytes)
                handles.append(c)
                caches.append(c)
                L.lab_gpu_enc_copy(stage, 0, c, 0, init.size)
            if min(handles) < 0 or L.lab_gpu_commit(1) != 1:
                raise RuntimeError("filling the KV caches failed")
        buf = {}
        for name, size in sizes.items():
            buf[name] = L.lab_gpu_buffer(4 * size)
            handles.append(buf[name])
        logits_h = L.lab_gpu_readback_buffer(4 * VOCAB)
        handles.append(logits_h)
        if min(handles) < 0:
            raise RuntimeError("lab_gpu_buffer failed")
        x_view = np.ctypeslib.as_array((ctypes.c_float * HIDDEN).from_address(L.lab_gpu_contents(buf["x"])))
        logits_view = np.ctypeslib.as_array(
            (ctypes.c_float * VOCAB).from_address(L.lab_gpu_contents(logits_h)))
        eps_bits = int(np.array([1e-6], np.float64).view(np.int64)[0])
        B = buf

        def norm(slot):
            return [2, B["x"], 0, small, 4 * HIDDEN * slot, B["a"], 0, 1, HIDDEN, eps_bits, 0]

        def add():
            return [4, B["m"], 0, B["x"], 0, HIDDEN, 0, 0, 0, 0, 0]


        def attention_block(layer, wqkv, aqkv):
            """As GpuForward records it (gpu.dart:1151-1175): q, k and v products
            (row ranges of the stacked qkv weights), k and v written straight
            into the caches' row `context`; q and k norm + RoPE in place; attention."""
            keys, values = caches[2 * layer], caches[2 * layer + 1]
            q_dim = HEADS * HEAD_DIM
            row = 4 * context * kv_dim

            def part(r0, rows, y, y_off):  # rows r0 .. r0 + rows of the stacked matrix
                return [0, wqkv, r0 * HIDDEN, aqkv + r0 * (HIDDEN // 32) * 4, B["a"], 0, y, y_off, rows,
                        HIDDEN, 1]

            def hnr(x, x_off, stride, heads, w_off):
                packed = heads | (HEAD_DIM << 16) | (1 << 32)
                return [7, x, x_off, stride, qk_norms, w_off, B["rope"], 0, 2 * HEAD_DIM, packed, eps_bits]

            return [part(0, q_dim, B["q"], 0),
                    part(q_dim, kv_dim, keys, row),
                    part(q_dim + kv_dim, kv_dim, values, row),
                    hnr(B["q"], 0, q_dim, HEADS, 4 * 2 * HEAD_DIM * layer),
                    hnr(keys, row, kv_dim, KV_HEADS, 4 * (2 * HEAD_DIM * layer + HEAD_DIM)),
                    [9, B["q"], keys, values, -1, B["attn"], context, 1, HEADS, KV_HEADS, HEAD_DIM]]

        table = []
        for layer in range(LAYERS):
            (wqkv, aqkv), (wo, ao), (wgu, agu), (wd, ad) = mats[4 * layer:4 * layer + 4]
            half_qs, half_sc = INTER * HIDDEN, INTER * (HIDDEN // 32) * 4
            o_in = "attn" if context > 0 else "qkv"
            table += [norm(2 * layer)]
            if context > 0:
                table += attention_block(layer, wqkv, aqkv)
            else:
                table += [[0, wqkv, 0, aqkv, B["a"], 0, B["qkv"], 0, OUT_ROWS["qkv"], HIDDEN, 1]]
            table += [[0, wo, 0, ao, B[o_in], 0, B["m"], 0, HIDDEN, HIDDEN, 1],
                      add(),
                      norm(2 * layer + 1),
                      [0, wgu, 0, agu, B["a"], 0, B["g"], 0, INTER, HIDDEN, 1],
                      [0, wgu, half_qs, agu + half_sc, B["a"], 0, B["u"], 0, INTER, HIDDEN, 1],
                      [3, B["g"], B["u"], INTER, 0, 0, 0, 0, 0, 0, 0],
                      [0, wd, 0, ad, B["g"], 0, B["m"], 0, HIDDEN, INTER, 1],
                      add()]
        wl, al = mats[-1]
        table += [norm(2 * LAYERS), [0, wl, 0, al, B["a"], 0, logits_h, 0, VOCAB, HIDDEN, 1]]
        table = np.ascontiguousarray(np.array(table, np.int64))
        x0 = stack.x0.cpu().numpy()
        rope_view = np.ctypeslib.as_array(
            (ctypes.c_float * (2 * HEAD_DIM)).from_address(L.lab_gpu_contents(B["rope"])))
        half = HEAD_DIM // 2
        angle = context / 1e6 ** (np.arange(half) * 2 / HEAD_DIM)
        rope_view[:] = np.concatenate([np.cos(angle), np.sin(angle), np.cos(angle), np.sin(angle)])

        def run(fused):
            L.dn_gpu_set_fusion(1 if fused else 0)
            dev_ms = []

            def one_token():
                x_view[:] = x0
                L.lab_gpu_begin()
                L.dn_gpu_enc_batch(table.ctypes.data, len(table))
                if L.lab_gpu_commit(1) != 1:
                    raise RuntimeError("lab_gpu_commit failed")
                dev_ms.append(L.lab_gpu_last_ms())

            for _ in range(3):
                one_token()
            dev_ms.clear()
            t0 = time.perf_counter()
            for _ in range(steps):
                one_token()
            tps = steps / (time.perf_counter() - t0)
            return tps, float(np.median(dev_ms)), logits_view.copy()

        fused_tps, fused_ms, fused_logits = run(True)
        plain_tps, plain_ms, plain_logits = run(False)
        L.dn_gpu_set_fusion(1)
        workload = (f"Qwen3-1.7B-shaped decode stack with its neighbours: {LAYERS} x [RMSNorm, "
                    "qkv, o, add, RMSNorm, gate, up, SwiGLU, down, add] + RMSNorm + lm_head "
                    "(attention omitted), batch 1, through lab_gpu_* with one "
                    "dn_gpu_enc_batch per token")
        if context > 0:
            workload = (f"Qwen3-1.7B-shaped decode step at position {context}: {LAYERS} x [RMSNorm, "
                        "q, k and v products (k and v into the KV caches' rows), q/k head norm + "
                        "RoPE, attention over the cache, o, add, RMSNorm, gate, up, SwiGLU, down, "
                        "add] + RMSNorm + lm_head, batch 1, as GpuForward records it, through "
                        "lab_gpu_* with one dn_gpu_enc_batch per token; KV caches device-resident "
                        "(dn_gpu_device_buffer)")
        return {
            "workload": workload,
            "ops_per_token": len(table),
            "fused": {"tokens_s": fused_tps, "commit_device_ms": fused_ms,
                      # with attention: q, k and v in one grouped launch, the q and k head
                      # norms in one launch, attention
                      "kernels_per_token": (4 + (2 if context > 0 else 0)) * LAYERS + 1,
                      "note": "the products only: each norm runs in the prologue of its first "
                              "reader, gate and up run as one dual GEMV with the SwiGLU in its "
                              "epilogue, the adds in the o and down epilogues; with attention, q, "
                              "k and v run as one grouped GEMV and their head norms as one launch"},
            "unfused": {"tokens_s": plain_tps, "commit_device_ms": plain_ms,
                        "kernels_per_token": (10 + (5 if context > 0 else 0)) * LAYERS + 2},  # the same
            "logits_identical": bool(np.array_equal(fused_logits.view(np.uint32),
                                                    plain_logits.view(np.uint32))),
            "logits_finite": bool(np.isfinite(fused_logits).all()),
            "steps": steps,
        }
    finally:
        L.dn_gpu_set_fusion(1)
        for h in handles:
            if h >= 0:
                L.lab_gpu_release(h)


def run_neighbours_workload(args):
    """Only the decode stack with its neighbours (run_neighbours), one JSON
    line; with --layers, a shorter stack for profiler captures."""
    import torch
    from dianoia_b200 import _lib
    L = _lib.lib()
    if L.lab_cpu_supported() != 1:
        raise SystemExit("no sm_100 device visible to libdianoia_b200")
    stack = Stack(torch, 0, 1, torch.device("cuda", 0))
    torch.cuda.synchronize()
    res = run_neighbours(args, stack, L)
    res["layers"] = LAYERS
    res["decode_step"] = run_neighbours(args, stack, L, context=args.context)
    print(json.dumps(res), flush=True)


def run_cache_workload(args):
    """The config-3 stack's weights as a Q8 cache file (lib/src/q8_cache.dart
    layout, written by dianoia_b200.q8_cache), brought into device memory two
    ways: (1) as dianoia's GpuForward does, mapping the file and wrapping the
    mapping (lab_gpu_wrap copies it into the buffer's host mirror; the first
    commit copies that to the device), timed up to a first product; (2)
    dn_gpu_wrap_file, reading the file straight into device memory through
    pinned staging. The file was just written, so its pages are in the page
    cache. One JSON line; both buffers give the same product, bit for bit."""
    import tempfile
    import torch
    from dianoia_b200 import _lib
    from dianoia_b200.q8_cache import Q8Cache
    L = _lib.lib()
    if L.lab_cpu_supported() != 1 or L.lab_gpu_init() != 1:
        raise SystemExit("no sm_100 device visible to libdianoia_b200")
    stack = Stack(torch, 0, 1, torch.device("cuda", 0))
    torch.cuda.synchronize()

    class Host:
        format = "q8"

        def __init__(self, m):
            self.rows, self.cols = m["rows"], m["cols"]
            self.qs_bytes = m["qs"].cpu().numpy().view(np.uint8)
            self.scale_bytes = m["scales"].cpu().numpy().view(np.uint8)

    tmp = tempfile.mkdtemp(prefix="dn_cache_")
    path = os.path.join(tmp, "stack.q8cache")
    names = [f"{i}.{m['name']}" for i, m in enumerate(stack.mats)]
    by_name = dict(zip(names, stack.mats))
    t0 = time.perf_counter()
    Q8Cache.write_each(path, "bench", [(n, "q8", by_name[n]["rows"], by_name[n]["cols"]) for n in names],
                       lambda n: Host(by_name[n]))
    write_s = time.perf_counter() - t0
    size = os.path.getsize(path)
    handles = []
    try:
        cache = Q8Cache.open(path, "bench")
        m0 = stack.mats[-1]  # the lm_head: a product to touch the weights
        o = cache.offsets(names[-1], m0["rows"], m0["cols"])
        act = L.lab_gpu_buffer(4 * HIDDEN)
        out = L.lab_gpu_readback_buffer(4 * VOCAB)
        handles += [act, out]
        x = np.ctypeslib.as_array((ctypes.c_float * HIDDEN).from_address(L.lab_gpu_contents(act)))
        x[:] = stack.x0.cpu().numpy()
        y = np.ctypeslib.as_array((ctypes.c_float * VOCAB).from_address(L.lab_gpu_contents(out)))

        def product(w):
            L.lab_gpu_begin()
            L.lab_gpu_enc_matmul_q8(w, o["qs"], o["scales"], act, 0, out, 0, m0["rows"], m0["cols"], 1)
            if L.lab_gpu_commit(1) != 1:
                raise RuntimeError("lab_gpu_commit failed")
            return y.copy()

        t0 = time.perf_counter()
        mapped = L.lab_gpu_wrap(cache.file.address, cache.file.length)
        handles.append(mapped)
        wrap_s = time.perf_counter() - t0
        y_mapped = product(mapped)
        mapped_s = time.perf_counter() - t0
        t0 = time.perf_counter()
        on_file = L.dn_gpu_wrap_file(path.encode(), 0, size)
        handles.append(on_file)
        file_s = time.perf_counter() - t0
        if min(mapped, on_file) < 0:
            raise RuntimeError("wrapping the cache failed")
        y_file = product(on_file)
        cache.close()
        res = {
            "workload": "Q8 cache of the config-3 stack (113 Q8_0 matrices, reference layout) "
                        "into device memory",
            "file_bytes": size, "write_s": write_s,
            "lab_gpu_wrap_of_mapping": {"s": mapped_s, "gbs": size / mapped_s / 1e9,
                                        "wrap_call_s": wrap_s,
                                        "note": "lab_gpu_wrap (copy into the pinned host mirror) "
                                                "+ the first commit's device copy and one product"},
            "dn_gpu_wrap_file": {"s": file_s, "gbs": size / file_s / 1e9,
                                 "note": "up to 8 host threads, each a contiguous slice through "
                                         "two 16 MiB pinned chunks (a device copy overlapping "
                                         "the next read); page-cache-hot file"},
            "products_identical": bool(np.array_equal(y_mapped.view(np.uint32), y_file.view(np.uint32))),
            "product_matches_stack": bool(np.array_equal(
                y_file.view(np.uint32), run_lm_head_reference(stack, L).view(np.uint32))),
        }
        print(json.dumps(res), flush=True)
    finally:
        for h in handles:
            if h >= 0:
                L.lab_gpu_release(h)
        os.remove(path)
        os.rmdir(tmp)


def run_lm_head_reference(stack, L):
    """The lm_head product of x0 on the device-resident stack (dn_linear)."""
    import torch
    m = stack.mats[-1]
    y = torch.empty(m["rows"], dtype=torch.float32, device=stack.device)
    xq = torch.empty(m["cols"], dtype=torch.int8, device=stack.device)
    xsc = torch.empty(m["cols"] // 32, dtype=torch.float32, device=stack.device)
    rc = L.dn_linear(0, m["qs"].data_ptr(), m["scales"].data_ptr(), stack.x0.data_ptr(),
                     xq.data_ptr(), xsc.data_ptr(), y.data_ptr(), m["rows"], m["cols"], 1, m["rows"],
                     1, -1, 0, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    if rc != 0:
        raise RuntimeError(f"dn_linear failed: {rc}")
    return y.cpu().numpy()


def run_cpu_baseline(args, stack):
    from oracle import oracle as orc
    bind_cpu_threads()
    try:
        ref = orc.Reference()
        kind = "reference"
    except FileNotFoundError:
        return None
    hw = host_weights(stack)
    x0 = stack.x0.cpu().numpy()
    threads = host_threads()
    cpu_reference_tokens(ref, hw, x0, threads, 1)  # warm-up (page-in, OpenMP pool)
    sec, logits = cpu_reference_tokens(ref, hw, x0, threads, args.cpu_tokens)
    same = bool(np.array_equal(logits, stack.bufs["lm_head"].cpu().numpy()))
    # The same stack on one thread (one token: a bounded sample).
    sec1, logits1 = cpu_reference_tokens(ref, hw, x0, 1, 1)
    return {"value": 1.0 / sec, "unit": "tokens/s", "cores": threads, "kind": kind,
            "cpu_model": cpu_model(), "omp_proc_bind": os.environ.get("OMP_PROC_BIND", "unset"),
            "threads_1": {"value": 1.0 / sec1, "unit": "tokens/s", "sample": "1 token, 1 thread",
                          "logits_bit_identical_to_gpu": bool(np.array_equal(logits1, logits))},
            "sample": f"{args.cpu_tokens} tokens of the full stack (113 lab_gemm_q8 mode-1 calls "
                      f"each, OpenMP, OMP_PROC_BIND={os.environ.get('OMP_PROC_BIND', 'unset')})",
            "logits_bit_identical_to_gpu": same}


if __name__ == "__main__":
    main()
