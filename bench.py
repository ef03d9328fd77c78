"""HCA decode benchmark (BASELINE config 2 per GPU, through the 37-layer HCA stack).

A step is one decode step of the HCA layer path for 64 requests x 3 query
tokens (ECHO/MTP with 2 drafts) at contexts U[4096, 131072], fp8 KV, 64
heads x 128: per-step metadata build, then for each of 37 HCA layers (each
with its own caches and inputs, so L2 cannot serve repeats) the Q head-norm +
RoPE with the fp8 SWA insert, compressor state save + block compression,
sparse attention over [window || compressed] rows, and VHA + inverse RoPE +
FP8 quant.  The input GEMMs and wo_a / wo_b are outside the path.  The step is
captured in one CUDA graph.

Multi-GPU (torchrun): requests shard data-parallel, 64 per GPU, no
collective (weak scaling); timing is the max over ranks of the device time.

``--impl reference`` times the reference's CPU restatement of the same path
(the oracle port) on the host cores; rank 0 only.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "vllm-ernie_b200"))

import numpy as np  # noqa: E402
import torch  # noqa: E402

LAYERS = 37
BATCH = 64
Q_PER_SEQ = 3
CTX_LO, CTX_HI = 4096, 131072
MAX_COMPRESSED = 1024  # ceil(131072 / 128) rounded to 128
METRIC = "HCA attn tokens/s & HBM roofline % (decode, 128K ctx, fp8 KV) at 1/2/4/8 B200"
UNIT = "tokens/s"


def peaks() -> tuple[float, str]:
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def tensor_peak() -> tuple[float, str]:
    """Dense bf16 TFLOP/s: the burst figure (a kernel timed alone)."""
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            return float(json.load(f)["bf16_tflops"]), "measured"
    except Exception:
        return 1590.0, "fallback"


def attention_flops(ctx: np.ndarray, heads: int, head_dim: int) -> int:
    """sum over query tokens of H * rows(t) * 4 D, rows(t) = (p+1)//128 +
    min(p+1, 128): the two GEMMs (S = Q K^T, O = P V) of one attention launch."""
    p = (ctx[:, None] + np.arange(Q_PER_SEQ)[None, :]).reshape(-1)
    rows = (p + 1) // 128 + np.minimum(p + 1, 128)
    return int(rows.sum()) * heads * 4 * head_dim


def contexts(rank: int) -> np.ndarray:
    rng = np.random.default_rng(1234 + rank)
    return rng.integers(CTX_LO, CTX_HI - Q_PER_SEQ, size=BATCH, endpoint=True)


# config 4: 16 sequences whose last query is at position ~1,048,575 (8192
# compressed entries plus the 128-token window each), 3 queries per sequence
BATCH_1M, CTX_1M, MAX_COMPRESSED_1M = 16, 1048573, 8320


def contexts_1m(rank: int) -> np.ndarray:
    rng = np.random.default_rng(4321 + rank)
    return CTX_1M - rng.integers(0, 128, size=BATCH_1M)


def row_bytes_algo(head_dim: int, rope_dim: int = 64) -> int:
    """Bytes of one cached row: N e4m3 + 2R bf16 + N/64 scales (N = D - R)."""
    nope = head_dim - rope_dim
    return nope + 2 * rope_dim + nope // 64


def algorithmic_bytes(ctx: np.ndarray, heads: int, head_dim: int) -> int:
    """Unique KV rows read + Q read + O write of one attention launch."""
    last = ctx + Q_PER_SEQ - 1
    rows = (last + 1) // 128 + np.minimum(last + 1, 128 + Q_PER_SEQ - 1)
    t = len(ctx) * Q_PER_SEQ
    return int(rows.sum()) * row_bytes_algo(head_dim) + 2 * t * heads * head_dim * 2


class ClockSampler:
    """NVML samples of the SM clock and the clock-event reasons, every 2 ms,
    during the timed region (read only: no setting of the GPU is touched)."""

    # nvmlClocksEventReason bits
    REASONS = {"sw_power_cap": 0x4, "hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40}

    def __init__(self, index: int):
        self.index = index
        self.samples: list[tuple[float, int]] = []
        self.max_mhz = None
        self.stop = threading.Event()
        self.handle = None

    def _open(self):
        import pynvml

        pynvml.nvmlInit()
        try:
            pr = torch.cuda.get_device_properties(self.index)
            bus = f"{pr.pci_domain_id:08x}:{pr.pci_bus_id:02x}:{pr.pci_device_id:02x}.0"
            h = pynvml.nvmlDeviceGetHandleByPciBusId(bus)
        except Exception:
            h = pynvml.nvmlDeviceGetHandleByIndex(self.index)
        self.max_mhz = float(pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM))
        return pynvml, h

    def _run(self):
        nv, h = self.nv, self.handle
        while not self.stop.is_set():
            try:
                mhz = float(nv.nvmlDeviceGetClockInfo(h, nv.NVML_CLOCK_SM))
                reasons = int(nv.nvmlDeviceGetCurrentClocksEventReasons(h))
                self.samples.append((mhz, reasons))
            except Exception:
                break
            time.sleep(0.002)

    def __enter__(self):
        try:
            self.nv, self.handle = self._open()
            self.t = threading.Thread(target=self._run, daemon=True)
            self.t.start()
        except Exception:
            self.handle = None
        return self

    def __exit__(self, *a):
        self.stop.set()
        if self.handle is not None:
            self.t.join(timeout=5)

    def summary(self) -> dict:
        sm = [m for m, _ in self.samples]
        seen = set()
        for _, r in self.samples:
            for name, bit in self.REASONS.items():
                if r & bit:
                    seen.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": self.max_mhz,
                "reasons": sorted(seen), "samples": len(sm), "source": "nvml, 2 ms"}


def setup_dist(cpu_only: bool = False):
    """One process per GPU (NCCL); the CPU-only reference arm uses gloo and
    touches no GPU."""
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    import datetime

    if cpu_only:
        if ws > 1:
            torch.distributed.init_process_group("gloo", timeout=datetime.timedelta(seconds=600))
        return ws, rank, local
    torch.cuda.set_device(local)
    if ws > 1:
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                             device_id=torch.device("cuda", local))
    return ws, rank, local


def barrier(ws):
    if ws > 1:
        torch.distributed.barrier()


def max_over_ranks(x: float, ws: int) -> float:
    if ws == 1:
        return x
    t = torch.tensor([x], device="cuda", dtype=torch.float64)
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return float(t.item())


# ---------------------------------------------------------------------------
# CPU arm: the oracle port of the same path
# ---------------------------------------------------------------------------


_CPU_FIXTURES: dict = {}


def _cpu_worker(job) -> tuple[int, float]:
    """One process of the CPU baseline: the oracle over requests
    worker, worker + n_workers, ... for ~budget seconds, one BLAS thread."""
    worker, n_workers, budget = job
    from threadpoolctl import threadpool_limits

    torch.set_num_threads(1)
    with threadpool_limits(limits=1):
        tokens, t, _ = _cpu_sample(budget, worker, n_workers)
    return tokens, t


def cpu_pool(processes: int | None = None):
    """The CPU baseline's worker pool (spawn: safe after CUDA use)."""
    import concurrent.futures as cf
    import multiprocessing as mp

    n = processes or os.cpu_count() or 1
    return cf.ProcessPoolExecutor(max_workers=n, mp_context=mp.get_context("spawn")), n


def cpu_sample_tokens_per_s(seconds_budget: float = 15.0, pool=None) -> dict:
    """The oracle (CPU restatement of the reference path) on all host cores:
    a spawn-context process pool, each worker timing whole config-2 requests
    (3 query tokens) through one layer's Q prep, SWA insert, compressor,
    sparse attention and VHA/inverse RoPE with one BLAS thread; the workers'
    rates add up.  Tokens/s are scaled to the 37-layer step."""
    own = pool is None
    ex, n = cpu_pool() if own else pool
    try:
        res = list(ex.map(_cpu_worker, [(w, n, seconds_budget) for w in range(n)]))
    finally:
        if own:
            ex.shutdown()
    rate = sum(tok / t for tok, t in res if t > 0)
    tokens = sum(tok for tok, _ in res)
    return {"value": rate / LAYERS, "unit": UNIT, "cores": n, "kind": "port",
            "sample": f"{tokens // Q_PER_SEQ} config-2 requests x {Q_PER_SEQ} tokens through one HCA layer on {n} "
                      f"processes (~{seconds_budget:.0f} s each, one BLAS thread each), scaled to the "
                      f"{LAYERS}-layer step"}


def _cpu_sample(seconds_budget: float, worker: int = 0, n_workers: int = 1) -> tuple[int, float, int]:
    from oracle import attention as A
    from oracle import cache as C
    from oracle import metadata as M
    from oracle import output as O

    ctx = contexts(0)
    heads, d, r = 64, 128, 64
    cos_sin = C.rope_cos_sin_cache(CTX_HI + 8, r, 160000.0)

    def fixture(b: int):
        """Request b's inputs and compact caches (built once, reused): SWA
        pages only for the window, compressor-state pages only for the 128
        positions a block boundary pools, every compressed entry."""
        if b in _CPU_FIXTURES:
            return _CPU_FIXTURES[b]
        rng = np.random.default_rng(7 + b)
        L = int(ctx[b])
        end = L + Q_PER_SEQ
        ncomp = end // 128 + 1

        def compact_pages(lo: int, page: int):
            first, last = lo // page, (end - 1) // page
            bt = np.zeros((1, (end + page - 1) // page), np.int32)
            bt[0, first:last + 1] = np.arange(last - first + 1)
            return bt, last - first + 1

        swa_bt, n_swa = compact_pages(max(L - 127, 0), 64)
        swa = np.zeros((n_swa, C.page_bytes(64, d, r)), np.uint8)
        live = np.arange(max(L - 127, 0), L)
        live_slots = swa_bt[0, live // 64] * 64 + live % 64
        C.insert_rows(swa, live_slots, rng.standard_normal((len(live), d)).astype(np.float32), 64, d, r)
        comp = np.zeros(((ncomp + 1) // 2 + 1, C.page_bytes(2, d, r)), np.uint8)
        C.insert_rows(comp, np.arange(ncomp), rng.standard_normal((ncomp, d)).astype(np.float32), 2, d, r)
        comp_bt = np.arange(comp.shape[0], dtype=np.int32)[None]
        st_bt, n_st = compact_pages(max(L - 128, 0), 8)
        state = rng.standard_normal((n_st, 8, 2 * d)).astype(np.float32)
        q = rng.standard_normal((Q_PER_SEQ, heads, d)).astype(np.float32)
        kv = rng.standard_normal((Q_PER_SEQ, d)).astype(np.float32)
        ks = rng.standard_normal((Q_PER_SEQ, 2 * d)).astype(np.float32)
        _CPU_FIXTURES[b] = (L, end, swa, swa_bt, comp, comp_bt, state, st_bt, q, kv, ks)
        return _CPU_FIXTURES[b]

    done_tokens, t_total, reqs = 0, 0.0, 0
    wall0 = time.perf_counter()
    mine = list(range(worker, len(ctx), n_workers)) or [worker % len(ctx)]
    for it in range(100 * len(ctx)):
        b = mine[it % len(mine)]
        L, end, swa, swa_bt, comp, comp_bt, state, st_bt, q, kv, ks = fixture(b)
        pos = np.arange(L, end)
        qsl = np.array([0, Q_PER_SEQ], np.int32)
        sl = np.array([end], np.int32)
        t0 = time.perf_counter()
        qp = O.q_prep(q, pos, cos_sin, r, 1e-6)
        swa_slot = M.slot_mapping(qsl, sl, swa_bt, 64)
        C.insert_rows(swa, swa_slot, O.kv_rope(kv, pos, cos_sin, r), 64, d, r)
        st_slot = M.slot_mapping(qsl, sl, st_bt, 8)
        C.save_partial_states(state, ks[:, :d], ks[:, d:], np.zeros((128, d), np.float32), pos, st_slot, 8, 128)
        t2r = np.zeros(Q_PER_SEQ, np.int32)
        c_slot = M.compressed_slot_mapping(Q_PER_SEQ, qsl, sl, comp_bt, 2, 128)
        C.compress_norm_rope_store(state, t2r, pos, st_slot, st_bt, 8, np.ones(d, np.float32), 1e-6, cos_sin,
                                   comp, c_slot, 2, d, r)
        idx = np.zeros((Q_PER_SEQ, 128), np.int32)
        lens = np.zeros(Q_PER_SEQ, np.int32)
        M.swa_indices_and_lens(Q_PER_SEQ, 128, qsl, sl, t2r, swa_slot >= 0, swa_bt, 64, idx, lens)
        gd = np.zeros((Q_PER_SEQ, MAX_COMPRESSED), np.int32)
        dl = np.zeros(Q_PER_SEQ, np.int32)
        M.c128a_topk_metadata(pos, 128, Q_PER_SEQ, t2r, comp_bt, 2, swa_slot, gd, dl,
                              np.zeros((1, MAX_COMPRESSED), np.int32), MAX_COMPRESSED)
        o = A.sparse_decode(qp, swa, 64, idx, lens, comp, 2, gd, dl, d ** -0.5, np.zeros(heads, np.float32), d, r)
        mix = np.eye(heads, dtype=np.float32)
        O.inv_rope_fp8_quant(np.einsum("hg,tgd->thd", mix, o), pos, cos_sin, 8, r)
        t_total += time.perf_counter() - t0
        done_tokens += Q_PER_SEQ
        reqs += 1
        # bounded in CPU time of the timed ops and in wall time (fixture builds)
        if t_total > seconds_budget or time.perf_counter() - wall0 > 3 * seconds_budget + 30:
            break
    return done_tokens, t_total, reqs


L2_NOTE = "inputs larger than L2: every layer has its own caches, cycled each step (run.l2 gives the bytes)"


def decode_config(ws: int, layers: int, tokens: int, long_ctx: bool = False, head_dim: int = 128) -> dict:
    """The workload keys of a decode line; both arms print the same dict."""
    if long_ctx:
        wl = (f"config 4 (16 req x 3 q at ~1M context: 8192 compressed + 128 window rows, H=64, D={head_dim}, "
              f"fp8 KV) x {layers} HCA layers")
    elif head_dim == 512:
        wl = (f"config 2 requests at the model's head_dim (64 req x 3 q, ctx U[4K,128K], H=64, D=512, fp8 KV) "
              f"x {layers} HCA layers")
    else:
        wl = f"config 2 (64 req x 3 q, ctx U[4K,128K], H=64, D=128, fp8 KV) x {layers} HCA layers"
    return {"workload": wl, "parallelism": f"dp{ws}", "layers": layers, "tokens_per_step_per_gpu": tokens,
            "l2": L2_NOTE}


def run_reference(args, ws, rank):
    if rank != 0:
        return
    sys.path.insert(0, ROOT)
    for _ in range(args.warmup):
        pass
    vals = []
    budget = max(3.0, 20.0 / max(args.steps, 1))
    pool = cpu_pool()
    try:
        for _ in range(max(args.steps, 1)):
            vals.append(cpu_sample_tokens_per_s(budget, pool))
    finally:
        pool[0].shutdown()
    v = statistics.median([x["value"] for x in vals])
    cb = dict(vals[0])
    cb["value"] = v
    line = {"metric": METRIC, "value": v, "unit": UNIT, "n_gpus": ws, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": Q_PER_SEQ * BATCH / v * 1e3,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic", "impl": "reference",
            "config": decode_config(ws, LAYERS, BATCH * Q_PER_SEQ),
            "run": {"where": "the oracle port on the host cores"},
            "cpu_baseline": cb,
            "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# prefill workload (config 3): a supplementary line, not the headline metric
# ---------------------------------------------------------------------------

PREFILL_SEQS, PREFILL_CHUNK = 8, 8192
PREFILL_METRIC = "HCA chunked-prefill tokens/s & tensor roofline % (8 x 8192-token chunks, prior 0-120K, fp8 KV)"


def prefill_contexts(rank: int) -> np.ndarray:
    rng = np.random.default_rng(4321 + rank)
    return 128 * rng.integers(0, 960, size=PREFILL_SEQS, endpoint=True)


def prefill_flops(ctx: np.ndarray, heads: int, head_dim: int, chunk: int = PREFILL_CHUNK) -> float:
    """Attention FLOPs of one layer: sum over query tokens of
    heads x rows x 4 D, rows = (p + 1) // 128 + min(p + 1, 128)."""
    tot = 0
    for c in ctx.tolist():
        p = np.arange(c, c + chunk, dtype=np.int64)
        tot += int(((p + 1) // 128 + np.minimum(p + 1, 128)).sum())
    return float(tot) * heads * 4 * head_dim


def run_prefill(args, ws, rank, local):
    from vllm_ernie_b200 import ops
    from vllm_ernie_b200.decode import build_prefill_metadata, prefill_layer, random_layer_weights
    from vllm_ernie_b200.synthetic import HCADims, alloc_layer_caches, make_decode_batch, rope_cos_sin_cache

    dev = torch.device("cuda", local)
    dims = HCADims(heads=64, head_dim=128, rope_dim=64, n_groups=8)
    ctx = prefill_contexts(rank)
    chunk = args.prefill_chunk
    batch = make_decode_batch(ctx.tolist(), chunk, dims, dev, seed=rank, max_model_len=CTX_HI)
    T = batch.num_tokens
    layers = args.layers if args.layers != LAYERS else 4
    caches = [alloc_layer_caches(batch, seed=20_000 * rank + l) for l in range(layers)]
    weights = [random_layer_weights(dims, dev, seed=l) for l in range(layers)]
    g = torch.Generator(device=dev).manual_seed(77 + rank)
    q_raw = [torch.randn((T, dims.heads, dims.head_dim), generator=g, device=dev).to(torch.bfloat16)
             for _ in range(layers)]
    kv = torch.randn((layers, T, dims.head_dim), generator=g, device=dev).to(torch.bfloat16)
    kv_score = torch.randn((layers, T, 2 * dims.head_dim), generator=g, device=dev)
    cos_sin = rope_cos_sin_cache(CTX_HI + chunk + 8, dims.rope_dim, dims.rope_theta, dev)
    bufs: dict = {}
    q_buf = torch.empty((T, dims.heads, dims.head_dim), dtype=torch.bfloat16, device=dev)
    o_buf = torch.empty_like(q_buf)

    def step():
        m = build_prefill_metadata(batch, buffers=bufs)
        for l in range(layers):
            prefill_layer(batch, m, caches[l], weights[l], q_raw[l], kv[l], kv_score[l], cos_sin, q_buf=q_buf,
                          o_buf=o_buf)

    step()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        step()
    torch.cuda.current_stream().wait_stream(s)
    with torch.cuda.graph(graph):
        step()
    for _ in range(max(args.warmup, 3)):
        graph.replay()
    torch.cuda.synchronize()
    barrier(ws)
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        torch.cuda.nvtx.range_push("prefill_step")  # profiler filter: the timed step replays
        ev0.record()
        for _ in range(args.steps):
            graph.replay()
        ev1.record()
        torch.cuda.nvtx.range_pop()
        torch.cuda.synchronize()
    barrier(ws)
    ms = max_over_ranks(ev0.elapsed_time(ev1) / args.steps, ws)

    # the attention launch alone, back to back over the layers
    md = build_prefill_metadata(batch, buffers=bufs)
    qs = [ops.fused_qnorm_rope_kv_insert(q_raw[l], kv[l], caches[l].swa, md.swa_slot, batch.positions, cos_sin,
                                         dims.heads, dims.eps, dims.swa_page, dims.rope_dim) for l in range(layers)]

    def attn_all():
        for l in range(layers):
            ops.sparse_prefill(qs[l], batch.query_start_loc, batch.seq_lens, caches[l].swa, dims.swa_page,
                               batch.swa_bt, caches[l].comp, dims.comp_page, batch.comp_bt, dims.window, dims.ratio,
                               dims.head_dim ** -0.5, weights[l].attn_sink, out=o_buf, rope_dim=dims.rope_dim)

    attn_all()
    torch.cuda.synchronize()
    ag = torch.cuda.CUDAGraph()
    with torch.cuda.stream(s):
        attn_all()
    torch.cuda.current_stream().wait_stream(s)
    with torch.cuda.graph(ag):
        attn_all()
    ag.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    reps = max(3, min(args.steps, 10))
    e0.record()
    for _ in range(reps):
        ag.replay()
    e1.record()
    torch.cuda.synchronize()
    attn_us = e0.elapsed_time(e1) * 1e3 / (reps * layers)

    # the streamed Q prep and VHA kernels alone, back to back over the layers
    # (each launch reads a 1 GB input: larger than L2)
    def graph_us(fn):
        fn()
        torch.cuda.synchronize()
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.stream(s):
            fn()
        torch.cuda.current_stream().wait_stream(s)
        with torch.cuda.graph(gr):
            fn()
        gr.replay()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(reps):
            gr.replay()
        b.record()
        torch.cuda.synchronize()
        del gr
        return a.elapsed_time(b) * 1e3 / (reps * layers)

    qprep_us = graph_us(lambda: [ops.fused_qnorm_rope_kv_insert(
        q_raw[l], kv[l], caches[l].swa, md.swa_slot, batch.positions, cos_sin, dims.heads, dims.eps, dims.swa_page,
        dims.rope_dim, out=q_buf) for l in range(layers)])
    vha_us = graph_us(lambda: [ops.vha_inv_rope_fp8_quant(
        o_buf, weights[l].vha_mix, batch.positions, cos_sin, dims.n_groups, dims.nope, dims.rope_dim)
        for l in range(layers)])
    hd, hh, rd = dims.head_dim, dims.heads, dims.rope_dim
    cache_row = (hd - rd) + 2 * rd + (hd - rd) // 64 + 1
    qprep_bytes = T * (2 * hh * hd * 2 + hd * 2 + rd * 4 + cache_row)
    vha_bytes = T * (hh * hd * 2 + hh * hd + hh * 4 + rd * 4)
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            hbm_peak = float(json.load(f)["hbm_gbs"])
    except Exception:
        hbm_peak = 6650.0
    streams = {k: {"us": us, "algorithmic_bytes": nb, "gbs": nb / (us * 1e-6) / 1e9,
                   "frac_hbm": nb / (us * 1e-6) / 1e9 / hbm_peak}
               for k, us, nb in (("qprep_stream_kernel", qprep_us, qprep_bytes),
                                 ("vha_stream_kernel", vha_us, vha_bytes))}
    flops = prefill_flops(ctx, dims.heads, dims.head_dim, chunk)
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            peak, src = float(json.load(f)["bf16_tflops"]), "measured (burst)"
    except Exception:
        peak, src = 1590.0, "fallback"
    achieved = flops / (attn_us * 1e-6) / 1e12
    if rank == 0:
        line = {
            "metric": PREFILL_METRIC, "value": ws * T / (ms * 1e-3), "unit": "tokens/s", "n_gpus": ws,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": f"config 3 (8 x {chunk}-token chunks, prior 128*U[0,960], H=64, D=128, fp8 KV) "
                                   f"x {layers} HCA layers", "parallelism": f"dp{ws}", "layers": layers,
                       "tokens_per_step_per_gpu": T, "per_layer_us": ms * 1e3 / layers,
                       "l2": f"inputs larger than L2 ({T * dims.heads * dims.head_dim * 2 / 2**30:.2f} GB of Q per layer)"},
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                         "frac": achieved / peak, "traffic": None, "peak_source": src,
                         "kernel": "hca_tc_attention_kernel<prefill>", "launch_us": attn_us,
                         "algorithmic_flops": flops},
            "streams": streams,
            "cpu_baseline": None, "e2e": None,
            "gpu_launches": (4 + 5 * layers) * args.steps,
            "clocks": clk.summary(),
        }
        print(json.dumps(line), flush=True)
    del graph, ag
    if ws > 1:
        torch.distributed.destroy_process_group()


# ---------------------------------------------------------------------------
# GPU arm
# ---------------------------------------------------------------------------


# ---------------------------------------------------------------------------
# the drop-in module: Ernie5_5HCAAttention.forward over the 37-layer stack
# ---------------------------------------------------------------------------


def module_forward_context(batch, layer, prefixes):
    """The step's forward context as the engine builds it: one CommonAttention
    metadata per cache group (SWA 64-token pages, compressed 256-token manager
    blocks, compressor state 8-token pages), the three builders, keyed by
    every layer's prefix."""
    from vllm_ernie_b200 import ops
    from vllm_ernie_b200.backend import (C128AMetadataBuilder, CommonAttentionMetadata, CompressorMetadataBuilder,
                                         HCAStepMetadata, SWAMetadataBuilder)

    dev = batch.device
    n = batch.num_tokens
    qsl, sl, pos = batch.query_start_loc, batch.seq_lens, batch.positions
    qsl_cpu = qsl.cpu()

    def common(bt, page):
        return CommonAttentionMetadata(query_start_loc=qsl, query_start_loc_cpu=qsl_cpu, seq_lens=sl,
                                       num_reqs=batch.num_reqs, num_actual_tokens=n, max_query_len=batch.q_per_seq,
                                       block_table_tensor=bt, slot_mapping=ops.slot_mapping(qsl, sl, bt, page, n),
                                       positions=pos, max_seq_len=int(batch.ctx.max()) + batch.q_per_seq)

    cm_swa = common(batch.swa_bt, batch.dims.swa_page)
    cm_comp = common(batch.comp_bt, batch.dims.comp_page * batch.dims.ratio)
    cm_st = common(batch.state_bt, batch.dims.state_page)
    spec = batch.q_per_seq - 1
    swa = SWAMetadataBuilder(batch.dims.window, max(n, 256), layer.n_local_heads, num_speculative_tokens=spec,
                             device=dev, head_dim=layer.head_dim).build(0, cm_swa)
    c128 = C128AMetadataBuilder(layer.max_model_len, max(n, 256), num_speculative_tokens=spec, device=dev).build(
        0, cm_comp, cm_swa.slot_mapping)
    comp = CompressorMetadataBuilder(max(n, 256), device=dev).build(0, cm_st)
    return HCAStepMetadata(swa, c128, comp).as_forward_context(prefixes)


def build_module_stack(batch, caches, layers: int, dev, seed: int = 0, tp_group=None):
    """``layers`` drop-in HCA modules of config 2's shape (hidden 4096, 64
    heads, q_lora 1024, 8 output groups of rank 1024) on the 128 x 128
    block-FP8 output path, random N(0, 0.02) weights (bf16 wo_a / wo_b
    block-quantised on load), bound to the bench's caches.  With a TP group
    every rank draws the same full weights and loads its head shard."""
    from vllm_ernie_b200 import attention as A

    d = batch.dims
    cfg = A.Ernie5_5HCAConfig(hidden_size=4096, num_hidden_layers=layers, num_attention_heads=d.heads,
                              head_dim=d.head_dim, q_lora_rank=1024, qk_rope_head_dim=d.rope_dim,
                              o_groups=d.n_groups, o_lora_rank=1024, hybrid_mla_num_attention_heads=d.heads,
                              num_nextn_predict_layers=0, compress_rope_theta=d.rope_theta)
    max_len = max(int(batch.ctx.max()) + batch.q_per_seq + 8, CTX_HI + 8)
    cfg.max_position_embeddings = max(cfg.max_position_embeddings, max_len)  # config 4 reaches ~1M positions
    vcfg = A.make_vllm_config(cfg, max_model_len=max_len, num_speculative_tokens=batch.q_per_seq - 1,
                              quant_config=A.block_fp8_quant_config())
    g = torch.Generator(device=dev).manual_seed(seed)
    aux = [torch.cuda.Stream(dev), torch.cuda.Stream(dev)]  # the model's aux streams, shared by the layers
    mods = []
    # full (unsharded) parameter shapes: those of a TP=1 layer
    full = {n: (p.shape, p.dtype) for n, p in
            A.Ernie5_5HCAAttention(vcfg, prefix="model.layers.shape_probe.self_attn").named_parameters()}
    for l in range(layers):
        m = A.Ernie5_5HCAAttention(vcfg, prefix=f"model.layers.{l}.self_attn", aux_stream_list=aux,
                                   tp_group=tp_group).to(dev)
        assert m.fp8_output
        ws = []
        for name, p in m.named_parameters():
            if name.endswith("weight_scale_inv"):
                continue
            shape = full[name][0]
            if name.endswith("norm.weight"):
                w = 1.0 + 0.02 * torch.randn(shape, generator=g, device=dev)
            elif name == "attn_sink":
                w = torch.randn(shape, generator=g, device=dev)
            else:
                w = 0.02 * torch.randn(shape, generator=g, device=dev)
            ws.append((name, w.to(torch.float32 if full[name][1] == torch.float32 else torch.bfloat16)))
        m.load_weights(ws)
        m.process_weights_after_loading()
        m.bind_kv_cache(caches[l].swa, caches[l].comp, caches[l].state)
        mods.append(m)
    return mods


def run_module(args, ws, batch, caches, layers, dev, attn_ms, tp_group=None):
    """Time the drop-in module: ``layers`` x ``Ernie5_5HCAAttention.forward``
    (input GEMMs, QK-norm, the attention op, the FP8 output GEMMs; a residual
    add feeds each layer's output to the next) captured in one CUDA graph,
    with the step's metadata built by the backend builders before it (as the
    engine does around its graphs).  Device-timed, and end to end: pinned
    host ``hidden_states`` and ``positions`` in, the last ``[T, hidden]`` out,
    copies inside the timed region."""
    from vllm_ernie_b200.forward_context import set_forward_context

    mods = build_module_stack(batch, caches, layers, dev, tp_group=tp_group)
    prefixes = [m.prefix for m in mods]
    T = batch.num_tokens
    ctx = module_forward_context(batch, mods[0], prefixes)
    g = torch.Generator(device=dev).manual_seed(7)
    hidden = torch.randn((T, 4096), generator=g, device=dev).to(torch.bfloat16)
    positions = batch.positions.clone()
    out = torch.empty_like(hidden)

    def step():
        h = hidden
        for m in mods:
            h = h + m(positions, h)
        out.copy_(h)

    with set_forward_context(ctx):
        step()
        torch.cuda.synchronize()
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            step()
        torch.cuda.current_stream().wait_stream(s)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            step()
    for _ in range(max(args.warmup, 3)):
        graph.replay()
    torch.cuda.synchronize()
    barrier(ws)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.nvtx.range_push("module_step")  # profiler filter: the timed module replays
    e0.record()
    for _ in range(args.steps):
        graph.replay()
    e1.record()
    torch.cuda.nvtx.range_pop()
    torch.cuda.synchronize()
    ms = max_over_ranks(e0.elapsed_time(e1) / args.steps, ws)
    assert torch.isfinite(out.float()).all(), "module output not finite"

    h_in = torch.empty(hidden.shape, dtype=hidden.dtype, pin_memory=True)
    h_pos = torch.empty(positions.shape, dtype=positions.dtype, pin_memory=True)
    h_out = torch.empty(out.shape, dtype=out.dtype, pin_memory=True)
    h_in.copy_(hidden)
    h_pos.copy_(positions)
    e2e_steps = max(3, min(args.steps, 10))
    barrier(ws)
    torch.cuda.synchronize()
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record()
    for _ in range(e2e_steps):
        hidden.copy_(h_in, non_blocking=True)
        positions.copy_(h_pos, non_blocking=True)
        graph.replay()
        h_out.copy_(out, non_blocking=True)
    t1.record()
    torch.cuda.synchronize()
    e2e_ms = max_over_ranks(t0.elapsed_time(t1) / e2e_steps, ws)
    del graph
    torch.cuda.synchronize()
    # per layer: q/kv RMSNorm, decode prep, attention, merge + VHA + inverse
    # RoPE + FP8 quant (TP: inverse RoPE + FP8 quant after the VHA
    # all-reduce), wo_a FP8 GEMM, gate quant, wo_b FP8 GEMM
    ours = 7 * layers
    tok = T if tp_group is not None else ws * T  # TP: every rank serves the same tokens
    return {
        "call": f"{layers} x Ernie5_5HCAAttention.forward(positions, hidden_states), block-FP8 wo_a/wo_b, one CUDA graph",
        "value": tok / (ms * 1e-3), "unit": UNIT, "ms_per_step": ms, "per_layer_us": ms * 1e3 / layers,
        "attention_share": attn_ms / ms if attn_ms else None,
        "gpu_launches_ours_per_step": ours,
    }, {
        "value": tok / (e2e_ms * 1e-3), "unit": UNIT,
        "h2d_bytes_per_step": h_in.numel() * h_in.element_size() + h_pos.numel() * h_pos.element_size(),
        "d2h_bytes_per_step": h_out.numel() * h_out.element_size(),
        "call": "the module stack above, hidden_states/positions from pinned host memory, output back",
    }


TP_METRIC = "HCA module decode tokens/s, head-sharded TP (config 2 requests on every rank)"


def run_tp(args, ws, rank, local):
    """Head-sharded TP (the config-5 variant): every rank serves the same 64
    requests x 3 tokens with 64 / N of the heads and output groups; the VHA
    low-rank term (fp32) and the wo_b output (bf16) are all-reduced over NCCL
    in every layer.  Strong scaling.  The all-reduces are also timed alone
    (the same sizes and count) for the collective's share of the step."""
    from vllm_ernie_b200.synthetic import HCADims, alloc_layer_caches, make_decode_batch

    dev = torch.device("cuda", local)
    dims = HCADims(heads=64, head_dim=128, rope_dim=64, n_groups=8)
    batch = make_decode_batch(contexts(0).tolist(), Q_PER_SEQ, dims, dev, seed=0, max_model_len=CTX_HI)
    T = batch.num_tokens
    layers = args.layers
    caches = [alloc_layer_caches(batch, seed=l) for l in range(layers)]
    group = torch.distributed.group.WORLD if ws > 1 else None
    with ClockSampler(local) as clk:
        module, e2e = run_module(args, ws, batch, caches, layers, dev, None, tp_group=group)
    coll = None
    if ws > 1:
        z = torch.zeros((T, 16, dims.head_dim), dtype=torch.float32, device=dev)
        y = torch.zeros((T, 4096), dtype=torch.bfloat16, device=dev)
        for _ in range(3):
            torch.distributed.all_reduce(z)
            torch.distributed.all_reduce(y)
        torch.cuda.synchronize()
        barrier(ws)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(layers):
            torch.distributed.all_reduce(z)
            torch.distributed.all_reduce(y)
        e1.record()
        torch.cuda.synchronize()
        ar_ms = max_over_ranks(e0.elapsed_time(e1), ws)
        coll = {"what": f"{layers} x (all-reduce fp32 [{T}, 16, {dims.head_dim}] + all-reduce bf16 [{T}, 4096]), NCCL",
                "ms_per_step_alone": ar_ms, "share_of_step": ar_ms / module["ms_per_step"]}
    if rank == 0:
        line = {"metric": TP_METRIC, "value": module["value"], "unit": UNIT, "n_gpus": ws, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": module["ms_per_step"], "higher_is_better": True,
                "scaling": "strong", "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
                "config": {"workload": (f"config 2 requests (64 req x 3 q, ctx U[4K,128K], H=64 sharded over "
                                        f"{ws}, D=128, fp8 KV) x {layers} HCA modules"),
                           "parallelism": f"tp{ws}", "layers": layers, "tokens_per_step_per_gpu": T, "l2": L2_NOTE},
                "module": module, "e2e": e2e, "collective": coll,
                "gpu_launches": module["gpu_launches_ours_per_step"] * args.steps, "clocks": clk.summary()}
        print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--parallel", default="dp", choices=["dp", "tp"],
                    help="dp: requests shard over the GPUs (the headline); tp: the module stack with the heads "
                         "sharded over the GPUs and NCCL all-reduces (a supplementary line)")
    ap.add_argument("--splits", type=int, default=0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--workload", default="decode", choices=["decode", "prefill", "decode1m"],
                    help="decode: the headline metric (config 2); prefill: config 3 and decode1m: config 4, "
                         "supplementary lines")
    ap.add_argument("--prefill-chunk", type=int, default=PREFILL_CHUNK,
                    help="tokens per sequence of the prefill workload (config 3: 8192; smaller for profiling)")
    ap.add_argument("--layers", type=int, default=LAYERS,
                    help="HCA layers per step (37 in the model; fewer only for profiler captures)")
    ap.add_argument("--items", type=int, default=0,
                    help="work-list items per step (0: one wave of CTAs, or of CTA pairs at head_dim 512)")
    ap.add_argument("--head-dim", type=int, default=128, choices=[128, 512],
                    help="128: config 2 (the headline); 512: the same decode at the model's own head size, "
                         "a supplementary line")
    args = ap.parse_args()
    ws, rank, local = setup_dist(cpu_only=args.impl == "reference")
    if args.impl == "reference":
        run_reference(args, ws, rank)
        if ws > 1:
            torch.distributed.destroy_process_group()
        return
    if args.workload == "prefill":
        run_prefill(args, ws, rank, local)
        return
    if args.parallel == "tp":
        run_tp(args, ws, rank, local)
        if ws > 1:
            torch.distributed.destroy_process_group()
        return

    from vllm_ernie_b200 import ops
    from vllm_ernie_b200.decode import build_decode_metadata, decode_layer, random_layer_weights
    from vllm_ernie_b200.synthetic import (HCADims, alloc_layer_caches, make_decode_batch,
                                           rope_cos_sin_cache)

    dev = torch.device("cuda", local)
    dims = HCADims(heads=64, head_dim=args.head_dim, rope_dim=64, n_groups=8)
    wide = args.head_dim == 512
    long_ctx = args.workload == "decode1m"
    ctx = contexts_1m(rank) if long_ctx else contexts(rank)
    ctx_hi = MAX_COMPRESSED_1M * 128 if long_ctx else CTX_HI
    maxc = MAX_COMPRESSED_1M if long_ctx else MAX_COMPRESSED
    batch = make_decode_batch(ctx.tolist(), Q_PER_SEQ, dims, dev, seed=rank, max_model_len=ctx_hi)
    T = batch.num_tokens
    layers = args.layers
    caches = [alloc_layer_caches(batch, seed=10_000 * rank + l) for l in range(layers)]
    weights = [random_layer_weights(dims, dev, seed=l) for l in range(layers)]
    g = torch.Generator(device=dev).manual_seed(99 + rank)
    q_raw = torch.randn((layers, T, dims.heads, dims.head_dim), generator=g, device=dev).to(torch.bfloat16)
    kv = torch.randn((layers, T, dims.head_dim), generator=g, device=dev).to(torch.bfloat16)
    kv_score = torch.randn((layers, T, 2 * dims.head_dim), generator=g, device=dev)
    cos_sin = rope_cos_sin_cache(ctx_hi + 8, dims.rope_dim, dims.rope_theta, dev)
    bufs: dict = {}
    splits = args.splits or None
    md = build_decode_metadata(batch, maxc, num_splits=splits, buffers=bufs, max_items=args.items or None)
    q_buf = torch.empty((T, dims.heads, dims.head_dim), dtype=torch.bfloat16, device=dev)
    o_buf = torch.empty_like(q_buf)
    outs = [None] * layers

    def step():
        m = build_decode_metadata(batch, maxc, num_splits=splits, buffers=bufs, max_items=args.items or None)
        for l in range(layers):
            outs[l] = decode_layer(batch, m, caches[l], weights[l], q_raw[l], kv[l], kv_score[l], cos_sin,
                                   q_buf=q_buf, o_buf=o_buf)

    # metadata: token->req, 2 slot maps, compressed slot map (fill + map),
    # window indices, C128A indices (+ the work list); per layer: the decode
    # prep (Q prep, KV insert, state save, compress), attention, then either
    # the fused split merge + VHA/inverse-RoPE/FP8 (scheduled, head_dim 128) or
    # the split merge (if any) and VHA/inverse-RoPE/FP8
    combine = md.schedule is not None or md.num_splits > 1
    per_layer = 3 if (md.schedule is not None and not wide) else (4 if combine else 3)
    launches_per_step = 7 + (1 if md.schedule is not None else 0) + layers * per_layer
    step()  # warm (allocations, workspace)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        step()
    torch.cuda.current_stream().wait_stream(s)
    with torch.cuda.graph(graph):
        step()
    for _ in range(max(args.warmup, 3)):
        graph.replay()
    torch.cuda.synchronize()

    barrier(ws)
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clk:
        torch.cuda.nvtx.range_push("decode_step")  # profiler filter: the timed step replays
        ev0.record()
        for _ in range(args.steps):
            graph.replay()
        ev1.record()
        torch.cuda.nvtx.range_pop()
        torch.cuda.synchronize()
    barrier(ws)
    ms = ev0.elapsed_time(ev1) / args.steps
    ms = max_over_ranks(ms, ws)
    value = ws * T / (ms * 1e-3)

    # --- dominant kernel: sparse attention, one launch per layer in a graph ---
    attn_graph = torch.cuda.CUDAGraph()
    qs = [torch.empty_like(q_buf) for _ in range(layers)]
    for l in range(layers):
        ops.fused_qnorm_rope_kv_insert(q_raw[l], kv[l], caches[l].swa, md.swa_slot, batch.positions, cos_sin,
                                       dims.heads, dims.eps, dims.swa_page, dims.rope_dim, out=qs[l])

    def attn_all():
        for l in range(layers):
            ops.sparse_decode(qs[l], caches[l].swa, dims.swa_page, md.swa_indices, md.swa_lens, caches[l].comp,
                              dims.comp_page, md.comp_indices, md.comp_lens, dims.head_dim ** -0.5,
                              weights[l].attn_sink, out=o_buf, group_starts=md.group_starts,
                              max_group_tokens=md.max_group_tokens, num_splits=md.num_splits,
                              schedule=md.schedule, max_items=md.max_items)

    attn_all()
    torch.cuda.synchronize()
    with torch.cuda.stream(s):
        attn_all()
    torch.cuda.current_stream().wait_stream(s)
    with torch.cuda.graph(attn_graph):
        attn_all()
    for _ in range(3):
        attn_graph.replay()
    torch.cuda.synchronize()
    reps = max(args.steps, 5)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(reps):
        attn_graph.replay()
    e1.record()
    torch.cuda.synchronize()
    attn_us = e0.elapsed_time(e1) * 1e3 / (reps * layers)
    algo = algorithmic_bytes(ctx, dims.heads, dims.head_dim)
    hbm, src = peaks()
    achieved = algo / (attn_us * 1e-6) / 1e9
    flops = attention_flops(ctx, dims.heads, dims.head_dim)
    tpk, tsrc = tensor_peak()
    tflops = flops / (attn_us * 1e-6) / 1e12
    traffic = None
    prof = os.path.join(ROOT, "profiles", "decode_attention_traffic.json")
    if os.path.exists(prof) and not wide and not long_ctx:
        try:
            with open(prof) as f:
                traffic = json.load(f).get("bytes_per_launch")
        except Exception:
            traffic = None

    # --- the drop-in module over the same caches; e2e through it ---
    module, e2e = run_module(args, ws, batch, caches, layers, dev, ms)

    cache_bytes = sum(t.numel() * t.element_size() for c in caches for t in (c.swa, c.comp, c.state))
    l2_note = (f"inputs larger than L2: {layers} layers' caches, {cache_bytes / 1e6:.0f} MB, cycled"
               if cache_bytes > 126e6 else f"caches {cache_bytes / 1e6:.0f} MB fit in L2 (profiling case only)")

    cpu = None
    if rank == 0 and ws == 1 and not args.no_cpu_baseline and not wide and not long_ctx:
        sys.path.insert(0, ROOT)
        cpu = cpu_sample_tokens_per_s(15.0)

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": ws, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": decode_config(ws, layers, T, long_ctx, dims.head_dim),
            "run": {"split_k": (f"balanced work list, {md.max_items} CTAs" if md.schedule is not None
                                else f"{md.num_splits} uniform splits per request"),
                    "l2": l2_note, "per_layer_us": ms * 1e3 / layers},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s",
                         "frac": achieved / hbm, "traffic": traffic, "peak_source": src,
                         "kernel": ("hca_wide_attention_kernel<decode> (CTA pairs)" if wide
                                    else "hca_tc_attention_kernel<decode>") + (" + split merge" if combine else ""),
                         "launch_us": attn_us,
                         "algorithmic_bytes": algo,
                         # decode is balanced between HBM and the tensor pipe (arithmetic intensity ~290
                         # FLOP/B at config 2): the same launch against the bf16 tensor peak
                         "tensor": {"achieved": tflops, "peak": tpk, "unit": "TFLOP/s", "frac": tflops / tpk,
                                    "flops": flops, "peak_source": tsrc}},
            "cpu_baseline": cpu,
            "e2e": e2e,
            "module": module,
            "gpu_launches": launches_per_step * args.steps,
            "clocks": clk.summary(),
        }
        print(json.dumps(line), flush=True)
    del graph, attn_graph
    if ws > 1:
        torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
