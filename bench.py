#!/usr/bin/env python
"""Benchmark of the quantized decode GEMV (ZeroLlm QuantizedKernels.MatVecMulQ8_0 /
ZeroTensor GgufDequantizer.GemvQ8_0) on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload: single Q8_0 linear 4096 x 4096 (out x in), x ~ N(0,1) fp32, W ~ N(0,0.02) quantized to Q8_0 in
blocks of 32 with fp16 scales, y fp32 [4096].  One step = one GEMV over each of R = 16 distinct weight
copies (286 MB in total, above the 126 MB L2, so every launch streams its weights from HBM).  At N > 1
every rank runs the same workload on its own GPU (replicas: the GEMV has no cross-rank exchange), and
`value` is the sum over ranks.

Prints one JSON line (rank 0).  `value` is device-timed weight-stream throughput with everything resident;
`e2e` is the same metric through the reference bridge entry zc_gemv_q8_0 with host (pinned) buffers, the
weight and activation copies to the device and the result copy back inside the timed region.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "quant-matmul weight GB/s (% HBM peak); decode tokens/s at 1/2/4/8 B200"
ROWS = COLS = 4096
N_COPIES = 16
QBYTES = ROWS * COLS + ROWS * (COLS // 32) * 2   # int8 values + fp16 scales streamed per launch
ALGO_BYTES = QBYTES + COLS * 4 + ROWS * 4        # + x read + y written
AOS_BYTES = ROWS * (COLS // 32) * 34             # the reference's packed weight bytes
# Published CPU figure for this exact GEMV (ZeroTensor/README.md:198-203): 3.79 ms for the 17.8 MB weight.
PUBLISHED_GBS = AOS_BYTES / 3.79e-3 / 1e9
# dram__bytes_read.sum + dram__bytes_write.sum of one gemv_slab_kernel launch of this workload (17,856,000 read +
# 0 written), from an ncu capture of this command; reported as the roofline's traffic with that source named.
NCU_TRAFFIC_BYTES = 17856000


def workload_config(world):
    """The workload both arms report (the GPU arm and the reference arm run the same one)."""
    return {"workload": f"q8_0_gemv_{ROWS}x{COLS}", "rows": ROWS, "cols": COLS, "weight_copies": N_COPIES,
            "step": f"one GEMV over each of the {N_COPIES} weight copies",
            "l2": f"inputs larger than L2: {N_COPIES} rotating weight copies, "
                  f"{N_COPIES * QBYTES / 1e6:.0f} MB", "parallelism": f"replicas x{world}"}


def _peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


class ClockSampler:
    """Polls NVML (the data nvidia-smi prints) every 20 ms on a background thread."""

    REASONS = {0x4: "sw_power_cap", 0x8: "hw_slowdown", 0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown",
               0x80: "hw_power_brake_slowdown", 0x2: "applications_clocks_setting", 0x10: "sync_boost"}

    def __init__(self, device_index: int):
        self.samples, self.reasons, self.max_mhz, self.ok = [], set(), None, False
        self._stop = threading.Event()
        try:
            import pynvml as N
            N.nvmlInit()
            h = None
            try:
                import torch
                uuid = str(torch.cuda.get_device_properties(device_index).uuid)
                h = N.nvmlDeviceGetHandleByUUID(("GPU-" + uuid) if not uuid.startswith("GPU-") else uuid)
            except Exception:
                h = N.nvmlDeviceGetHandleByIndex(device_index)
            self._N, self._h = N, h
            self.max_mhz = N.nvmlDeviceGetMaxClockInfo(h, N.NVML_CLOCK_SM)
            self.ok = True
        except Exception:
            self.ok = False

    def _run(self):
        N, h = self._N, self._h
        while not self._stop.is_set():
            try:
                self.samples.append(N.nvmlDeviceGetClockInfo(h, N.NVML_CLOCK_SM))
                r = N.nvmlDeviceGetCurrentClocksEventReasons(h)
                for bit, name in self.REASONS.items():
                    if r & bit:
                        self.reasons.add(name)
            except Exception:
                pass
            time.sleep(0.02)

    def __enter__(self):
        if self.ok:
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()
        return self

    def __exit__(self, *a):
        if self.ok:
            self._stop.set()
            self._t.join()

    def summary(self):
        if not self.ok or not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": sorted(self.reasons), "samples": 0}
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons), "samples": len(self.samples)}


# ----------------------------------------------------------------------------------------------------------
# CPU legs (the oracle restates the reference's C# MatVecMulQ8_0; test infrastructure used only here)
# ----------------------------------------------------------------------------------------------------------
def _cpu_weights(n_copies, seed=1234):
    import oracle as O
    rng = np.random.default_rng(seed)
    x = rng.standard_normal(COLS, dtype=np.float32)
    ws = [O.quantize_q8_0(rng.standard_normal((ROWS, COLS), dtype=np.float32) * np.float32(0.02))
          for _ in range(n_copies)]
    return ws, x


def cpu_baseline(seconds=10.0):
    """Times the oracle's MatVecMulQ8_0 (AVX2 order, one row per task, all host threads) on a bounded sample."""
    import oracle as O
    ws, x = _cpu_weights(8)
    y = np.empty(ROWS, np.float32)
    O.matvec(8, ws[0], x, ROWS, COLS, threads=0)
    calls, t0 = 0, time.perf_counter()
    while True:
        O.lib().orc_matvec_q8_0(ws[calls % 8].ctypes.data_as(O._u8p), x.ctypes.data_as(O._f32p),
                                y.ctypes.data_as(O._f32p), ROWS, COLS, 0, 0)
        calls += 1
        el = time.perf_counter() - t0
        if el >= seconds and calls >= 3:
            break
    gbs = calls * QBYTES / el / 1e9
    return {"value": round(gbs, 3), "unit": "GB/s", "cores": O.lib().orc_num_threads(), "kind": "port",
            "sample": f"{calls} calls of MatVecMulQ8_0 {ROWS}x{COLS} rotating 8 weight copies "
                      f"({8 * AOS_BYTES / 1e6:.0f} MB) in {el:.1f} s"}


def run_reference(args):
    """`--impl reference`: the reference's CPU path (the oracle's C++ restatement of the C#) on all host cores.
    Each step is what a GPU step is: one MatVecMulQ8_0 call on each of the 16 weight copies.  The K timed steps
    are repeated until at least --ref-min-s seconds have been timed (a 20-step region is ~80 ms on the CPU); value
    = weight bytes of every timed call / total timed seconds."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    import oracle as O
    ws, x = _cpu_weights(N_COPIES)
    y = np.empty(ROWS, np.float32)
    xp, yp = x.ctypes.data_as(O._f32p), y.ctypes.data_as(O._f32p)
    wps = [w.ctypes.data_as(O._u8p) for w in ws]

    def step():
        for w in wps:
            O.lib().orc_matvec_q8_0(w, xp, yp, ROWS, COLS, 0, 0)

    for _ in range(args.warmup):
        step()
    el, reps = 0.0, 0
    while reps == 0 or el < args.ref_min_s:
        t0 = time.perf_counter()
        for _ in range(args.steps):
            step()
        el += time.perf_counter() - t0
        reps += 1
    steps = args.steps * reps
    gbs = steps * N_COPIES * QBYTES / el / 1e9
    cores = O.lib().orc_num_threads()
    line = {"impl": "reference", "metric": METRIC, "value": round(gbs, 3), "unit": "GB/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(el / steps * 1e3, 4),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": round(gbs / PUBLISHED_GBS, 3),
            "dtype": "int8xfp32", "data": "synthetic (seeded N(0,0.02) weights, N(0,1) activations)",
            "config": workload_config(world),
            "execution": "host threads: C++ restatement of MatVecMulQ8_0 (AVX2 order, one row per task)",
            "timed_repeats": reps, "timed_s": round(el, 3),
            "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": cores, "kind": "port",
                             "sample": f"{reps} x {args.steps} steps of {N_COPIES} MatVecMulQ8_0 {ROWS}x{COLS} calls "
                                       f"({steps * N_COPIES} calls in {el:.2f} s; C++ restatement of the "
                                       "reference C#, AVX2 order, one row per task)"},
            "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------------------------------------------------
# Other configurations, reported beside the headline (same run, same GPU)
# ----------------------------------------------------------------------------------------------------------
def _peak_tflops():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["bf16_tflops"]), "measured bf16 dense (fp16 runs at the same rate)"
    except Exception:
        return 1590.0, "fallback"


def _cpu_loop(fn, seconds):
    """Calls fn() until `seconds` have passed (at least twice after one untimed call); returns (calls, seconds)."""
    fn()
    calls, t0 = 0, time.perf_counter()
    while True:
        fn()
        calls += 1
        el = time.perf_counter() - t0
        if el >= seconds and calls >= 2:
            return calls, el


def prefill_gemm_leg(dev, L, iters=20, with_cpu=False, cpu_tokens=64, cpu_s=5.0):
    """Batched prefill GEMM (the 512-token prefill workload): X fp32 [512, 4096] ~ N(0,1), W Q8_0 [11008, 4096]
    ~ N(0,0.02).  Device timing with X and Y resident; `e2e` adds the copy of X from pinned host memory and of Y
    back, every step; `cpu` is the oracle's PrefillPrompt loop (token-parallel MatVecMulQ8_0) on a bounded sample
    of the same tokens, checked against the device result for those tokens."""
    import torch
    from zeroplatform_b200.ops import QuantizedWeight, quantize
    M, N, K = 512, 11008, 4096
    g = torch.Generator(device=dev)
    g.manual_seed(7)
    blocks = quantize(8, torch.randn((N, K), generator=g, device=dev) * 0.02)
    w = QuantizedWeight.upload(8, blocks, N, K, device=dev)
    x = torch.randn((M, K), generator=g, device=dev)
    y = torch.empty((M, N), device=dev)
    s = torch.cuda.current_stream()

    def run():
        if L.zcu_gemm_q8_0(w.qs.data_ptr(), w.d.data_ptr(), x.data_ptr(), y.data_ptr(), M, N, K, 0, s.cuda_stream):
            raise RuntimeError("zcu_gemm_q8_0 failed")

    def timed(fn, n):
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(s)
        for _ in range(n):
            fn()
        e1.record(s)
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / n

    ms = timed(run, iters)
    flops = 2.0 * M * N * K
    peak, src = _peak_tflops()
    tf = flops / (ms * 1e-3) / 1e12
    status = L.zcu_device_status(1)
    hx = torch.empty((M, K), dtype=torch.float32, pin_memory=True)
    hx.copy_(x)
    hy = torch.empty((M, N), dtype=torch.float32, pin_memory=True)

    def e2e_call():
        x.copy_(hx, non_blocking=True)
        run()
        hy.copy_(y, non_blocking=True)

    ms_e2e = timed(e2e_call, max(3, iters // 2))
    out = {"ms": round(ms, 4), "tflops": round(tf, 1), "weight_GBs": round(w.nbytes / (ms * 1e-3) / 1e9, 1),
           "roofline": {"bound": "tensor", "achieved": round(tf, 1), "peak": peak, "unit": "TFLOP/s",
                        "frac": round(tf / peak, 3), "peak_source": src,
                        "what": "algorithmic 2*M*N*K / device time (the kernel issues three fp16 products per "
                                "k-step: hi/lo pairs of q*d and x)"},
           "e2e": {"value": round(flops / (ms_e2e * 1e-3) / 1e12, 1), "unit": "TFLOP/s", "ms": round(ms_e2e, 4),
                   "h2d_bytes_per_step": M * K * 4, "d2h_bytes_per_step": M * N * 4,
                   "api": "zcu_gemm_q8_0 with X copied from pinned host memory and Y copied back, every step"},
           "note": "tcgen05 kind::f16 on fp16 hi/lo pairs of q*d and x (three MMAs per k-step), fp32 "
                   "accumulate; includes the fp32 -> fp16 hi/lo activation conversion kernel", "device_status": status}
    if with_cpu:  # the oracle's PrefillPrompt loop on the first cpu_tokens tokens (test infrastructure)
        import oracle as O
        wb = np.ascontiguousarray(blocks.cpu().numpy())
        xs = np.ascontiguousarray(x[:cpu_tokens].cpu().numpy())
        ys = np.empty((cpu_tokens, N), np.float32)

        def cpu_call():
            O.lib().orc_matmul_q8_0(wb.ctypes.data_as(O._u8p), xs.ctypes.data_as(O._f32p),
                                    ys.ctypes.data_as(O._f32p), cpu_tokens, N, K, 0, 0)

        calls, el = _cpu_loop(cpu_call, cpu_s)
        ref = y[:cpu_tokens].cpu().numpy().astype(np.float64)
        err = float(np.max(np.abs(ys - ref)) / max(float(np.max(np.abs(ys))), 1e-30))
        out["cpu"] = {"value": round(2.0 * cpu_tokens * N * K * calls / el / 1e12, 4), "unit": "TFLOP/s",
                      "cores": O.lib().orc_num_threads(), "kind": "port",
                      "sample": f"{calls} passes of PrefillPrompt's token-parallel MatVecMulQ8_0 loop over "
                                f"{cpu_tokens} of the {M} tokens in {el:.1f} s (C++ restatement of the C#)",
                      "max_rel_err_vs_device": err}
    return out


def _model_12l(dev):
    """The 12-layer d768 model (12 heads x 64, SwiGLU 2048, vocab 32000), Q8_0 from seeded N(0,0.02)."""
    import numpy as np
    import torch
    from zeroplatform_b200.ops import quantize
    vocab, dim, layers, heads, ffn = 32000, 768, 12, 12, 2048
    g = torch.Generator(device=dev)
    g.manual_seed(11)

    def q8(rows, cols, n=None):
        shape = (rows, cols) if n is None else (n, rows, cols)
        return quantize(8, torch.randn(shape, generator=g, device=dev) * 0.02).cpu().numpy()

    return dict(vocab=vocab, dim=dim, layers=layers, heads=heads, kv_heads=heads, ffn=ffn, context_length=2048,
                eps=1e-5, rope_base=10000.0, tok_emb=q8(vocab, dim), lm_head=q8(vocab, dim), wq=q8(dim, dim, layers),
                wk=q8(dim, dim, layers), wv=q8(dim, dim, layers), wo=q8(dim, dim, layers), wgate=q8(ffn, dim, layers),
                wup=q8(ffn, dim, layers), wdown=q8(dim, ffn, layers),
                attn_norm=np.ones((layers, dim), np.float32), ffn_norm=np.ones((layers, dim), np.float32),
                final_norm=np.ones(dim, np.float32))


def serve_leg(dev, n_req=32, max_batch=16, n_new=64, seed=21):
    """Continuous batching on the 12-layer d768 model: n_req requests (prompts of 64-192 random ids, greedy, n_new
    tokens each) submitted at once to the engine's scheduler (zcu_engine_submit / zcu_engine_serve_step, max_batch
    rows): requests are admitted as rows free up and every step is one batched decode of all running requests.
    Against it, the same requests generated one after another (zcu_engine_generate: one kernel per token).  Both
    timed by the host clock around the whole run (each serve step synchronises), after a warm-up run of the same
    mix that captures the step graphs of every batch size."""
    import time
    import numpy as np
    from zeroplatform_b200.engine import LlmEngine
    m = _model_12l(dev)
    rng = np.random.default_rng(seed)
    prompts = [rng.integers(0, m["vocab"], int(n)).astype(np.int32) for n in rng.integers(64, 193, n_req)]
    per_seq = (192 + n_new) // 16 + 2
    e = LlmEngine(m, total_pages=max_batch * per_seq, page_size=16, max_batch=max_batch, max_pages_per_seq=per_seq,
                  max_prefill_tokens=192)

    def batched(id0):
        for i, p in enumerate(prompts):
            e.submit(id0 + i, p, n_new, temperature=0.0, top_k=1, top_p=1.0, repetition_penalty=1.0)
        done = toks = steps = 0
        t0 = time.perf_counter()
        while done < n_req:
            steps += 1
            for _, tok, fin, reason in e.serve_step():
                toks += int(tok >= 0 and reason != 1)
                done += int(fin)
        return toks, steps, time.perf_counter() - t0

    batched(1000)
    toks_b, steps_b, t_b = batched(2000)
    for i, p in enumerate(prompts[:2]):  # warm-up of the one-sequence path
        e.generate_greedy(5000 + i, p, n_new)
        e.free_sequence(5000 + i)
    toks_s = 0
    t0 = time.perf_counter()
    for i, p in enumerate(prompts):
        out, _, _ = e.generate_greedy(6000 + i, p, n_new)
        toks_s += len(out)
        e.free_sequence(6000 + i)
    t_s = time.perf_counter() - t0
    e.close()
    return {"requests": n_req, "max_batch": max_batch, "new_tokens_per_request": n_new,
            "prompt_tokens": int(sum(len(p) for p in prompts)), "generated_tokens": toks_b, "serve_steps": steps_b,
            "tok_s_batched": round(toks_b / t_b, 1), "tok_s_sequential": round(toks_s / t_s, 1),
            "speedup": round((toks_b / t_b) / (toks_s / t_s), 2), "batched_s": round(t_b, 3),
            "sequential_s": round(t_s, 3),
            "timing": "host wall clock around each whole run (prefills included), after a warm-up run"}


def decode_12l_leg(dev, with_cpu, n_prompt=512, n_new=128):
    """Small Llama decode workload: 12 layers, d 768, 12 heads x 64, SwiGLU 2048, vocab 32000, Q8_0 from N(0,0.02);
    512 random prompt ids then 128 greedy tokens (repetition penalty 1.0), 16-token fp16 KV pages."""
    import numpy as np
    from zeroplatform_b200.engine import LlmEngine
    m = _model_12l(dev)
    vocab, dim, layers, heads = m["vocab"], m["dim"], m["layers"], m["heads"]
    prompt = np.random.default_rng(5).integers(0, vocab, n_prompt).astype(np.int32)
    e = LlmEngine(m, total_pages=64, page_size=16, max_batch=1, max_pages_per_seq=64, max_prefill_tokens=n_prompt)
    e.generate_greedy(0, prompt, 8)            # warm-up: captures the decode-step graph
    e.free_sequence(0)
    toks, pre_ms, dec_ms = e.generate_greedy(1, prompt, n_new)
    e.close()
    # packed Q8_0 bytes streamed per decode token (every projection and the LM head; one embedding row)
    weight_bytes = sum(int(np.prod(m[k].shape)) for k in ("lm_head", "wq", "wk", "wv", "wo", "wgate", "wup", "wdown"))
    # K/V bytes read per decode token: every layer reads K and V (fp16) of its attended context; token i of the
    # n_new attends to n_prompt + i positions (the reference's last-layer length; one fewer below it, ignored)
    hd = dim // heads
    mean_ctx = n_prompt + (n_new - 1) / 2.0
    kv_bytes = layers * 2 * heads * hd * 2 * mean_ctx
    emb_bytes = dim // 32 * 34
    per_tok = weight_bytes + kv_bytes + emb_bytes
    tok_s = n_new / (dec_ms * 1e-3)
    peak, src = _peaks()
    gbs = per_tok * tok_s / 1e9
    out = {"prefill_ms": round(pre_ms, 3), "decode_ms": round(dec_ms, 3),
           "decode_tok_s": round(tok_s, 1), "us_per_token": round(dec_ms * 1e3 / n_new, 2),
           "prompt_tok_s": round(n_prompt / (pre_ms * 1e-3), 1),
           "tokens": int(len(toks)), "weight_bytes_per_token": int(weight_bytes),
           "kv_bytes_per_token_mean": int(kv_bytes),
           "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": peak, "unit": "GB/s",
                        "frac": round(gbs / peak, 3), "peak_source": src,
                        "what": "Q8_0 weights (every projection and the LM head) + mean K/V bytes + one embedding "
                                "row per decode token x tokens/s"}}
    if with_cpu:  # the oracle LlmEngine (C++ restatement of the reference C#) on the host cores, bounded sample
        import oracle as O
        ref = O.Engine(m, total_pages=64, page_size=16)
        t0 = time.perf_counter()
        logits = ref.prefill(1, prompt[:64], 0)
        t1 = time.perf_counter()
        n_cpu = 16
        tok = int(np.argmax(logits))
        for i in range(n_cpu):
            logits = ref.forward_token(1, tok, 64 + i)
            tok = int(np.argmax(logits))
        t2 = time.perf_counter()
        ref.close()
        out["cpu"] = {"value": round(n_cpu / (t2 - t1), 2), "unit": "tok/s",
                      "decode_tok_s": round(n_cpu / (t2 - t1), 2), "prompt_tok_s": round(64 / (t1 - t0), 2),
                      "cores": O.lib().orc_num_threads(), "kind": "port",
                      "sample": f"oracle LlmEngine: 64-token prompt then {n_cpu} greedy decode steps (context 64-80)"}
    return out

def decode_7b_leg(dev, rank, world, batch=32, n_ctx=2048, n_new=128, n_warm=3, layers=32, with_cpu=False,
                  cpu_layers=2, cpu_ctx=256, cpu_steps=8):
    """Tensor-parallel 7B decode workload: Llama-2-7B-shaped decoder (32 layers, d 4096, 32 heads, FFN 11008, vocab 32000, Q8_0
    from N(0,0.02)), decode batch 32, each sequence with a 2048-token context in 16-token fp16 pages, then 128
    greedy tokens per sequence; tensor parallel over the `world` GPUs of this job (one engine per rank).

    Weights are drawn on the device from one seed per tensor (the same full tensor on every rank, each rank
    keeps its slice) and quantized by zcu_quantize_q8_0.  The 2048-token contexts are written as synthetic
    N(0,1) K/V with zcu_engine_append_kv (PagedKvCache.AppendTokenAt) instead of being prefilled: the decode
    step reads the same pages either way, and a 65,536-token prefill is not part of this metric."""
    import torch
    import torch.distributed as dist
    from zeroplatform_b200.engine import LlmEngine, nccl_unique_id
    from zeroplatform_b200.ops import quantize
    vocab, dim, heads, ffn = 32000, 4096, 32, 11008
    hd = dim // heads
    model = dict(vocab=vocab, dim=dim, layers=layers, heads=heads, kv_heads=heads, ffn=ffn, context_length=4096)
    uid = None
    if world > 1:
        t = torch.zeros(128, dtype=torch.uint8, device=dev)
        if rank == 0:
            t.copy_(torch.frombuffer(bytearray(nccl_unique_id()), dtype=torch.uint8))
        dist.broadcast(t, 0)
        uid = bytes(t.cpu().numpy().tobytes())
    pages = (n_ctx + n_new + 15) // 16
    e = LlmEngine(model, total_pages=batch * pages, page_size=16, max_batch=batch, max_pages_per_seq=pages,
                  max_prefill_tokens=batch, tp_size=world, tp_rank=rank, nccl_id=uid, load=False)
    g = torch.Generator(device=dev)

    def q8(seed, rows, cols):
        g.manual_seed(seed)
        return quantize(8, torch.randn((rows, cols), generator=g, device=dev) * 0.02)

    t0 = time.perf_counter()
    host = {}  # the first cpu_layers layers' packed blocks for the CPU slice (rank 0 of a one-GPU run)
    cpu_layers = min(cpu_layers, layers)
    for name, seed in (("tok_emb", 1), ("lm_head", 2)):
        blk = q8(seed, vocab, dim)
        e.set_weight(name, 0, blk)
        if with_cpu:
            host[name] = blk.cpu().numpy()
    shapes = {"wq": (dim, dim), "wk": (dim, dim), "wv": (dim, dim), "wo": (dim, dim), "wgate": (ffn, dim),
              "wup": (ffn, dim), "wdown": (dim, ffn)}
    for layer in range(layers):
        for j, (name, (r, c)) in enumerate(shapes.items()):
            blk = q8(1000 + 10 * layer + j, r, c)
            e.set_weight(name, layer, blk)
            if with_cpu and layer < cpu_layers:
                host.setdefault(name, []).append(blk.cpu().numpy())
    t_weights = time.perf_counter() - t0
    # synthetic contexts: n_ctx - n_warm tokens per sequence (warm-up steps bring them to n_ctx)
    n_fill = n_ctx - n_warm
    for layer in range(layers):
        g.manual_seed(50000 + layer)
        k = torch.randn((n_fill, heads, hd), generator=g, device=dev).half()
        v = torch.randn((n_fill, heads, hd), generator=g, device=dev).half()
        for sid in range(batch):
            e.append_kv(sid, layer, 0, k, v)
    torch.cuda.synchronize()
    toks = np.random.default_rng(9).integers(0, vocab, batch).astype(np.int32)
    out, _ = e.generate_batch(list(range(batch)), toks, n_warm)           # captures the step graph
    out, ms = e.generate_batch(list(range(batch)), out[:, -1], n_new)
    if world > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    sh = e.shard()
    e.close()
    step_s = ms * 1e-3 / n_new
    # bytes one rank streams per step: its Q8_0 weight slice (SoA int8 + fp16 scales) and its K/V heads
    w_rank = layers * ((3 * sh["heads"] * hd + 2 * sh["ffn"]) * dim + dim * (sh["heads"] * hd + sh["ffn"])) \
        + sh["vocab"] * dim
    w_rank = w_rank * 34 // 32
    mean_ctx = n_ctx + (n_new + 1) / 2.0
    kv_rank = batch * mean_ctx * layers * 2 * sh["kv_heads"] * hd * 2
    peak, src = _peaks()
    gbs = (w_rank + kv_rank) / step_s / 1e9
    cpu = None
    if with_cpu:  # the oracle LlmEngine on a reduced slice of the same weights (test infrastructure)
        import oracle as O
        m = dict(vocab=vocab, dim=dim, layers=cpu_layers, heads=heads, kv_heads=heads, ffn=ffn, context_length=4096,
                 eps=1e-5, rope_base=10000.0, tok_emb=host["tok_emb"], lm_head=host["lm_head"],
                 attn_norm=np.ones((cpu_layers, dim), np.float32), ffn_norm=np.ones((cpu_layers, dim), np.float32),
                 final_norm=np.ones(dim, np.float32))
        for name in shapes:
            m[name] = np.stack(host[name])
        ref = O.Engine(m, total_pages=(cpu_ctx + cpu_steps) // 16 + 2, page_size=16)
        prompt = np.random.default_rng(9).integers(0, vocab, cpu_ctx).astype(np.int32)
        logits = ref.prefill(0, prompt, 0)
        tok = int(np.argmax(logits))
        t1 = time.perf_counter()
        for i in range(cpu_steps):
            tok = int(np.argmax(ref.forward_token(0, tok, cpu_ctx + i)))
        el = time.perf_counter() - t1
        ref.close()
        cpu = {"value": round(cpu_steps / el, 3), "unit": "tok/s", "cores": O.lib().orc_num_threads(),
               "kind": "port", "ms_per_token_slice": round(el / cpu_steps * 1e3, 2),
               "sample": f"oracle LlmEngine on a reduced slice: {cpu_layers} of {layers} layers (LM head and "
                         f"embedding in full), 1 sequence, {cpu_ctx}-token context, {cpu_steps} greedy decode "
                         f"steps; the full step ({layers} layers x batch {batch} x {n_ctx}-token contexts) is "
                         "infeasible on the CPU"}
    return {"decode_tok_s": round(batch * n_new / (ms * 1e-3), 1), "ms_per_step": round(ms / n_new, 4),
            "n_gpus": world, "parallelism": f"tp{world}", "layers": layers, "batch": batch, "context_at_start": n_ctx,
            "new_tokens": n_new, "weight_bytes_per_step_per_gpu": int(w_rank),
            "kv_bytes_per_step_per_gpu": int(kv_rank),
            "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(gbs / peak, 3), "peak_source": src,
                         "what": "weights + K/V one rank streams per step / device step time"},
            "setup_s": round(t_weights, 2),
            "data": "synthetic: weights N(0,0.02) -> Q8_0 on device; contexts are N(0,1) fp16 K/V written with "
                    "zcu_engine_append_kv, not prefilled; greedy tokens from random first ids",
            "timing": "device events around 128 replays of the captured batch step (NCCL all-reduces inside), "
                      "max over ranks", "cpu": cpu}


def moe_leg(dev, rank, world, iters=10, tokens=256, n_experts=8, top_k=2, dim=4096, ffn=14336, with_cpu=False,
            cpu_s=5.0):
    """Expert-parallel MoE workload: MoE FFN layer, 8 experts x SwiGLU FFN 14336 at d_model 4096, Q4_0 (group 32, fp16 scales)
    from N(0,0.02); 256 tokens of N(0,1) activations, router logits N(0,1), softmax over the top 2.  Expert
    parallel over the `world` GPUs of this job: each rank holds n_experts / world experts and 256 / world of the
    tokens; rows travel to the experts' ranks and back by NCCL all-to-all.  Timing: device events around the
    layer's forward (routing, dispatch, experts, return, combine), max over ranks."""
    import torch
    import torch.distributed as dist
    from zeroplatform_b200.engine import nccl_unique_id
    from zeroplatform_b200.moe import SparseMoeLayer
    from zeroplatform_b200.ops import quantize
    uid = None
    if world > 1:
        t = torch.zeros(128, dtype=torch.uint8, device=dev)
        if rank == 0:
            t.copy_(torch.frombuffer(bytearray(nccl_unique_id()), dtype=torch.uint8))
        dist.broadcast(t, 0)
        uid = bytes(t.cpu().numpy().tobytes())
    t_local = tokens // world
    s = torch.cuda.current_stream()
    m = SparseMoeLayer(n_experts, top_k, dim, ffn, qtype=4, max_tokens=t_local, ep_size=world, ep_rank=rank,
                       nccl_id=uid, stream=s.cuda_stream)
    g = torch.Generator(device=dev)
    per = n_experts // world
    host = {"gate": [], "up": [], "down": []}  # packed Q4_0 blocks for the CPU leg (one-GPU runs)
    for e in range(rank * per, (rank + 1) * per):  # other ranks' experts are ignored by set_expert anyway
        for j, (name, (r, c)) in enumerate((("gate", (ffn, dim)), ("up", (ffn, dim)), ("down", (dim, ffn)))):
            g.manual_seed(7000 + 10 * e + j)
            blk = quantize(4, torch.randn((r, c), generator=g, device=dev) * 0.02)
            m.set_expert(e, name, blk)
            if with_cpu:
                host[name].append(blk.cpu().numpy().reshape(-1))
    g.manual_seed(99 + rank)
    x = torch.randn((t_local, dim), generator=g, device=dev)
    logits = torch.randn((t_local, n_experts), generator=g, device=dev)
    res = torch.zeros((t_local, dim), device=dev)
    m.forward(x, res, logits)  # one forward from a zero residual: the values the CPU leg checks
    res_once = res.cpu().numpy()
    for _ in range(2):
        m.forward(x, res, logits)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(s)
    for _ in range(iters):
        m.forward(x, res, logits)
    e1.record(s)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / iters
    if world > 1:
        tt = torch.tensor([ms], device=dev)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        ms = float(tt.item())
    m.close()
    w_bytes = n_experts * 3 * dim * ffn * 18 // 32  # Q4_0 weight bytes of all experts (each rank reads its share)
    peak, src = _peaks()
    gbs_rank = (w_bytes / world) / (ms * 1e-3) / 1e9
    flops = 2.0 * tokens * top_k * 3 * dim * ffn
    cpu = None
    if with_cpu:  # the oracle's SparseMoeLayer.Forward token by token on a bounded sample (test infrastructure)
        import oracle as O
        eg, eu, ed = (np.ascontiguousarray(np.concatenate(host[k])) for k in ("gate", "up", "down"))
        xs, lg = x.cpu().numpy(), logits.cpu().numpy()
        n_done, worst = 0, 0.0
        t0 = time.perf_counter()
        while n_done < t_local and (n_done < 2 or time.perf_counter() - t0 < cpu_s):
            r = np.zeros(dim, np.float32)
            O.moe_forward(xs[n_done], 4, eg, eu, ed, dim, ffn, n_experts, top_k, r, router_logits=lg[n_done])
            worst = max(worst, float(np.max(np.abs(r - res_once[n_done])) / max(float(np.max(np.abs(r))), 1e-30)))
            n_done += 1
        el = time.perf_counter() - t0
        cpu = {"value": round(n_done / el, 2), "unit": "tokens/s", "ms_per_layer_256_tokens":
               round(el / n_done * tokens * 1e3, 1), "cores": O.lib().orc_num_threads(), "kind": "port",
               "sample": f"SparseMoeLayer.Forward (C++ restatement) for {n_done} of the {tokens} tokens, one at a "
                         f"time, in {el:.1f} s", "max_rel_err_vs_device": worst}
    return {"ms": round(ms, 4), "tokens_per_s": round(tokens / (ms * 1e-3), 1), "n_gpus": world,
            "parallelism": f"ep{world}", "tokens": tokens, "experts": n_experts, "top_k": top_k, "dim": dim,
            "ffn": ffn, "weight_bytes": w_bytes, "tflops": round(flops / (ms * 1e-3) / 1e12, 1),
            "roofline": {"bound": "hbm", "achieved": round(gbs_rank, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(gbs_rank / peak, 3), "peak_source": src,
                         "what": "Q4_0 expert weight bytes one rank streams per forward / device time"},
            "data": "synthetic: experts N(0,0.02) -> Q4_0 on device, x and router logits N(0,1)", "cpu": cpu}


# ----------------------------------------------------------------------------------------------------------
# GPU arm
# ----------------------------------------------------------------------------------------------------------
def run_ours(args):
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=120))

    from zeroplatform_b200 import _lib
    from zeroplatform_b200.ops import QuantizedWeight, quantize

    L = _lib.lib()
    gen = torch.Generator(device=dev)
    gen.manual_seed(1234 + rank)
    weights = []
    for _ in range(N_COPIES):
        w32 = torch.randn((ROWS, COLS), generator=gen, device=dev, dtype=torch.float32) * 0.02
        weights.append(QuantizedWeight.upload(8, quantize(8, w32), ROWS, COLS, device=dev))
        del w32
    x = torch.randn(COLS, generator=gen, device=dev, dtype=torch.float32)
    ys = torch.empty((N_COPIES, ROWS), device=dev, dtype=torch.float32)
    stream = torch.cuda.Stream(device=dev)

    def step():
        for r, w in enumerate(weights):
            rc = L.zcu_gemv_q8_0(w.qs.data_ptr(), w.d.data_ptr(), x.data_ptr(), ys[r].data_ptr(), ROWS, COLS, 0,
                                 stream.cuda_stream)
            if rc != 0:
                raise RuntimeError(f"zcu_gemv_q8_0 failed: {rc}")

    with torch.cuda.stream(stream):
        step()  # sets kernel attributes outside capture
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            step()

    def barrier():
        if world > 1:
            dist.barrier()

    sampler = ClockSampler(local)
    # graph.replay() launches on torch's current stream: every replay and both events go to `stream`
    with sampler, torch.cuda.stream(stream):
        # clock soak: the timed region of a short run lasts about a millisecond, less than the sampler's period, so
        # the GPU is first kept busy for --clock-soak-s (replays reported as clock_soak_replays); then exactly W
        # warm-up steps
        t_w = time.perf_counter()
        n_soak = 0
        while time.perf_counter() - t_w < args.clock_soak_s:
            graph.replay()
            n_soak += 1
            if n_soak % 200 == 0:
                stream.synchronize()
        for _ in range(args.warmup):
            graph.replay()
        stream.synchronize()
        barrier()
        torch.cuda.synchronize()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(args.steps):
            graph.replay()
        e1.record(stream)
        torch.cuda.synchronize()
        barrier()
    ms = e0.elapsed_time(e1)
    if world > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    ms_per_step = ms / args.steps
    launches = args.steps * N_COPIES
    per_rank_gbs = launches * QBYTES / (ms * 1e-3) / 1e9
    value = per_rank_gbs * world
    launch_s = ms * 1e-3 / launches
    achieved = ALGO_BYTES / launch_s / 1e9
    peak, peak_kind = _peaks()

    # End to end through the reference bridge entry zc_gemv_q8_0 with host buffers, every copy inside the
    # timed region.  Two forms: (a) weights registered once with zc_register_weights (they stay resident;
    # each call copies x in and y out and synchronises), (b) unregistered: each call also copies the
    # 17.8 MB weight over PCIe, as a bridge without residency would.
    def e2e_leg():
        host_w = [torch.empty(AOS_BYTES, dtype=torch.uint8, pin_memory=True) for _ in range(N_COPIES)]
        for hw in host_w:
            w32 = torch.randn((ROWS, COLS), generator=gen, device=dev, dtype=torch.float32) * 0.02
            hw.copy_(quantize(8, w32).reshape(-1))
        hx = torch.empty(COLS, dtype=torch.float32, pin_memory=True)
        hx.copy_(x)
        hy = torch.empty(ROWS, dtype=torch.float32, pin_memory=True)

        def e2e_step():
            for hw in host_w:
                rc = L.zc_gemv_q8_0(hw.data_ptr(), hx.data_ptr(), hy.data_ptr(), ROWS, COLS)
                if rc != 0:
                    raise RuntimeError(f"zc_gemv_q8_0 failed: {rc}")

        def timed(n):
            for _ in range(2):
                e2e_step()
            barrier()
            t0 = time.perf_counter()
            for _ in range(n):
                e2e_step()
            el = time.perf_counter() - t0
            if world > 1:
                t = torch.tensor([el], device=dev, dtype=torch.float64)
                dist.all_reduce(t, op=dist.ReduceOp.MAX)
                el = float(t.item())
            return el

        n_copy = max(2, min(args.steps, 10))
        el_copy = timed(n_copy)
        for hw in host_w:
            if L.zc_register_weights(8, hw.data_ptr(), ROWS, COLS) != 0:
                raise RuntimeError("zc_register_weights failed")
        n_res = max(3, min(args.steps, 200))
        el_res = timed(n_res)
        for hw in host_w:
            L.zc_unregister_weights(hw.data_ptr())
        res = {"value": round(n_res * N_COPIES * QBYTES * world / el_res / 1e9, 3), "unit": "GB/s",
               "h2d_bytes_per_step": N_COPIES * COLS * 4, "d2h_bytes_per_step": N_COPIES * ROWS * 4,
               "api": "zc_gemv_q8_0 with host buffers, weights registered once (zc_register_weights)",
               "calls": n_res * N_COPIES, "us_per_call": round(el_res / (n_res * N_COPIES) * 1e6, 2)}
        copy = {"value": round(n_copy * N_COPIES * QBYTES * world / el_copy / 1e9, 3), "unit": "GB/s",
                "h2d_bytes_per_step": N_COPIES * (AOS_BYTES + COLS * 4), "d2h_bytes_per_step": N_COPIES * ROWS * 4,
                "api": "zc_gemv_q8_0 with host buffers, weights copied every call"}
        return res, copy

    try:
        e2e, e2e_copy = e2e_leg()
    except Exception as ex:  # keep the device-timed line even if an e2e leg fails
        e2e, e2e_copy = {"value": None, "unit": "GB/s", "error": str(ex)[:200]}, None

    extra = {}
    if not args.no_extra:
        with_cpu = rank == 0 and world == 1 and not args.no_cpu
        try:
            extra["prefill_gemm_512x11008x4096"] = prefill_gemm_leg(dev, L, with_cpu=with_cpu)
        except Exception as ex:
            extra["prefill_gemm_512x11008x4096"] = {"error": str(ex)[:200]}
        try:
            extra["decode_12l_d768"] = decode_12l_leg(dev, with_cpu)
        except Exception as ex:
            extra["decode_12l_d768"] = {"error": str(ex)[:200]}
        try:
            extra["serve_12l_d768_32req"] = serve_leg(dev)
        except Exception as ex:
            extra["serve_12l_d768_32req"] = {"error": str(ex)[:200]}
        try:
            extra[f"decode_7b_b32_tp{world}"] = decode_7b_leg(dev, rank, world, layers=args.layers,
                                                              n_new=args.new_tokens, with_cpu=with_cpu)
        except Exception as ex:
            extra[f"decode_7b_b32_tp{world}"] = {"error": str(ex)[:300]}
        try:
            extra[f"moe_8x14336_top2_ep{world}"] = moe_leg(dev, rank, world, with_cpu=with_cpu)
        except Exception as ex:
            extra[f"moe_8x14336_top2_ep{world}"] = {"error": str(ex)[:300]}
    cpu = cpu_baseline() if (rank == 0 and world == 1 and not args.no_cpu) else None
    if rank == 0:
        line = {"metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "clock_soak_replays": n_soak, "ms_per_step": round(ms_per_step, 6),
                "higher_is_better": True, "scaling": "weak", "vs_baseline": round(value / PUBLISHED_GBS, 2),
                "dtype": "int8xfp32",
                "data": "synthetic (seeded N(0,0.02) weights quantized on device, N(0,1) activations)",
                "config": workload_config(world),
                "execution": f"one CUDA graph of {N_COPIES} GEMV launches (programmatic dependent launch) per step",
                "pct_hbm_peak": round(100.0 * per_rank_gbs / peak, 1),
                "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                             "frac": round(achieved / peak, 3), "peak_source": peak_kind,
                             "traffic": NCU_TRAFFIC_BYTES,
                             "traffic_source": "ncu dram__bytes_read.sum + dram__bytes_write.sum of one launch of "
                                               "this kernel on this workload (a capture of this command, not this run)",
                             "algorithmic_bytes_per_launch": ALGO_BYTES,
                             "kernel": "gemv_slab_kernel<XPlain>", "launch_us": round(launch_s * 1e6, 3)},
                "e2e": e2e, "e2e_weights_copied_per_call": e2e_copy, "gpu_launches": launches,
                "clocks": sampler.summary(), "cpu_baseline": cpu, "extra_configs": extra}
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def gemm_leg(dev, m, n, k, iters=5):
    """One Q8_0 tensor-core GEMM shape alone (seeded N(0,0.02) weights, N(0,1) activations), `iters` calls of
    zcu_gemm_q8_0 timed together -- the small command the GEMM profiles capture."""
    import torch
    from zeroplatform_b200 import _lib
    from zeroplatform_b200.ops import QuantizedWeight, quantize
    L = _lib.lib()
    g = torch.Generator(device=dev)
    g.manual_seed(1)
    w = QuantizedWeight.upload(8, quantize(8, torch.randn((n, k), generator=g, device=dev) * 0.02), n, k, device=dev)
    x = torch.randn((m, k), generator=g, device=dev)
    y = torch.empty((m, n), device=dev)
    s = torch.cuda.current_stream()

    def call():
        if L.zcu_gemm_q8_0(w.qs.data_ptr(), w.d.data_ptr(), x.data_ptr(), y.data_ptr(), m, n, k, 0, s.cuda_stream):
            raise RuntimeError("zcu_gemm_q8_0 failed")
    call()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(s)
    for _ in range(iters):
        call()
    e1.record(s)
    torch.cuda.synchronize()
    us = e0.elapsed_time(e1) * 1e3 / iters
    return {"us": round(us, 2), "tflops": round(2.0 * m * n * k / us / 1e6, 1),
            "weight_GBs": round(w.nbytes / us / 1e3, 1), "device_status": L.zcu_device_status(1)}


def run_leg(args):
    """`--leg decode_7b` / `--leg moe` / `--leg gemm --shape M,N,K`: one extra leg alone, printed as its own JSON
    line (rank 0).  --layers / --new-tokens shrink the decode leg for profiler captures."""
    import torch
    import torch.distributed as dist
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=120))
    if args.leg == "moe":
        res = moe_leg(dev, rank, world)
        name = f"moe_8x14336_top2_ep{world}"
    elif args.leg == "decode_12l":
        res = decode_12l_leg(dev, False)
        name = "decode_12l_d768"
    elif args.leg == "serve":
        res = serve_leg(dev)
        name = "serve_12l_d768_32req"
    elif args.leg == "gemm":
        m, n, k = (int(v) for v in args.shape.split(","))
        res = gemm_leg(dev, m, n, k)
        name = f"gemm_q8_0_{m}x{n}x{k}"
    else:
        res = decode_7b_leg(dev, rank, world, n_new=args.new_tokens, layers=args.layers)
        name = f"decode_7b_b32_tp{world}"
    if rank == 0:
        print(json.dumps({"leg": name, **res}), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--leg", choices=["all", "decode_7b", "decode_12l", "moe", "gemm", "serve"], default="all",
                    help="all: the headline and every extra leg; decode_7b: only the 7B tensor-parallel decode; serve: "
                         "continuous batching on the 12-layer model; "
                         "moe: only the expert-parallel MoE layer; gemm: one GEMM shape (--shape)")
    ap.add_argument("--shape", default="512,11008,4096", help="gemm: M,N,K")
    ap.add_argument("--layers", type=int, default=32, help="decode_7b: decoder layers (32 = the 7B shape)")
    ap.add_argument("--new-tokens", type=int, default=128, help="decode_7b: generated tokens per sequence")
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline leg")
    ap.add_argument("--no-extra", action="store_true", help="skip the prefill-GEMM and decoder legs")
    ap.add_argument("--clock-soak-s", type=float, default=1.0,
                    help="keep the GPU busy this long before the warm-up steps (clock samples under load)")
    ap.add_argument("--ref-min-s", type=float, default=2.0,
                    help="reference arm: repeat the K timed steps until at least this many seconds are timed")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    elif args.leg in ("decode_7b", "decode_12l", "moe", "gemm", "serve"):
        run_leg(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
