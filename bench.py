#!/usr/bin/env python
"""Benchmark of the B200 quantized-Llama decode path (decode tokens/s and weight-stream GB/s, b = 1).

Workload (the configuration the reference's headline metric is quoted
on): TinyLlama-1.1B-architecture, Q4_K_M, batch 1, greedy; 32-token seeded
prompt, 128 new tokens. A "step" is one generation's decode phase: 127
single-token decode steps after the prompt's prefill.

  value  decode tokens/s, device-timed (CUDA events around back-to-back
         launches of the persistent decode kernel, one per token; the
         prompt's prefill between steps is not timed), summed over ranks /
         max rank time.
  e2e    the same metric through the C ABI call (armai_llama_generate) with
         host buffers: prompt H2D, every token D2H to the host for the stop
         check, measured the way the reference measures it
         ((n_new - 1) / decode_us, llama_candle.rs:106-130, llama_candle.ex:99).

N > 1 (torchrun): independent replicas, one per GPU (batch-1 TinyLlama does
not shard; scaling "weak"). `--impl reference` times the reference's CPU
path (the oracle restatement of candle's generic kernels, all host threads)
on rank 0.
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "decode tokens/s and weight-stream HBM GB/s (% peak), Q4_K_M Llama, b=1"
ARCH = "tinyllama-1.1b"
PROMPT, MAX_NEW = 32, 128
PUBLISHED_TOK_S = 4.71  # the reference's published TinyLlama 1.1B Q4_K_M b=1 decode rate (Snapdragon 632)


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=5)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", default="armai", choices=["armai", "reference"])
    p.add_argument("--no-cpu-baseline", action="store_true", help="skip the CPU baseline sample")
    p.add_argument("--no-clocks", action="store_true")
    p.add_argument("--no-config2", action="store_true", help="skip the batched-decode (config 2) figures")
    p.add_argument("--no-config3", action="store_true", help="skip the Mistral-7B long-context (config 3) figures")
    p.add_argument("--no-config4", action="store_true", help="skip the Llama-3-8B tensor-parallel (config 4) figures")
    p.add_argument("--no-config5", action="store_true", help="skip the primitive sweep (config 5) figures")
    p.add_argument("--trace-decode", action="store_true",
                   help="print the per-phase timeline of one persistent-kernel decode step (globaltimer "
                        "stamps per CTA, armai_llama_trace_decode) after a 32-token prompt, instead of the bench")
    p.add_argument("--profile", default=None, choices=sorted(PROFILE_CASES),
                   help="run one case for a profiler instead of the bench: once untimed, then once between "
                        "cudaProfilerStart / Stop (ncu --profile-from-start off captures only that run)")
    return p.parse_args()


def _profile_case(name):
    """The cases the committed ncu summaries under profiles/ were captured on."""
    import ctypes
    import torch
    from arm_ai_b200 import native, synth
    from arm_ai_b200._lib import load_cuda
    path = synth.model_path(ARCH, seed=0)
    if name == "prefill512":  # one 512-token prompt through the tensor-core GEMMs and attention
        m = native.llama_candle_load_op(path, prefill_gemm=2, max_seq_len=2048)
        prompt = synth.prompt_tokens(512, 32000, 11)
        run = lambda: native.llama_forward(m, prompt, 0, want_logits=False)
    elif name == "batch16":  # 16 one-token prompts, then batched GEMM decode steps
        m = native.llama_candle_load_op(path, max_batch=16, max_seq_len=1024, batch_gemm=2)
        prompts = [synth.prompt_tokens(1, 32000, 50 + i) for i in range(16)]
        run = lambda: native.llama_generate_batch(m, prompts, 3)
    elif name == "batch16ctx512":  # 16 512-token prompts, then batched GEMM decode steps (config 2's context)
        m = native.llama_candle_load_op(path, max_batch=16, max_seq_len=1024, batch_gemm=2)
        prompts = [synth.prompt_tokens(512, 32000, 50 + i) for i in range(16)]
        run = lambda: native.llama_generate_batch(m, prompts, 3)
    elif name == "decode":  # one persistent-kernel decode step after a 32-token prompt
        m = native.llama_candle_load_op(path, max_seq_len=1024)
        native.llama_forward(m, synth.prompt_tokens(PROMPT, 32000, 3), 0, want_logits=False)
        pos = [PROMPT]
        def run():
            native.llama_forward(m, [5], pos[0], want_logits=False)
            pos[0] += 1
    else:  # config-5 primitives through the device-pointer entry points
        lib = load_cuda()
        dev = torch.device("cuda:0")
        P = lambda t: ctypes.c_void_p(t.data_ptr())
        if name == "attn2048":
            H, S, D = 32, 2048, 128
            q, k, v = (torch.rand(1, H, S, D, device=dev).half() * 2 - 1 for _ in range(3))
            o = torch.empty(1, H, S, D, device=dev)
            run = lambda: lib.armai_dev_flash_attention_f16(P(q), P(k), P(v), P(o), ctypes.c_float(D ** -0.5), 1, H,
                                                            S, S, D, 1, None)
        else:  # int8m512
            M, K = 512, 4096
            a = torch.randint(-127, 128, (M, K), dtype=torch.int8, device=dev)
            w = torch.randint(-127, 128, (K, K), dtype=torch.int8, device=dev)
            o = torch.empty(M, K, dtype=torch.int32, device=dev)
            run = lambda: lib.armai_dev_int8_matmul_s32(P(a), P(w), P(o), M, K, K, None)
    run()
    torch.cuda.synchronize()
    torch.cuda.profiler.start()
    run()
    torch.cuda.synchronize()
    torch.cuda.profiler.stop()


PROFILE_CASES = ("prefill512", "batch16", "batch16ctx512", "decode", "attn2048", "int8m512")


def _trace_decode(d):
    """Per-phase timeline of one decode step: per phase kind, the median over
    layers of (the phase's median end over CTAs - the previous phase's),
    the phase's own median duration and its activation-build time; then one
    middle layer's slot medians relative to the phase start (slots: 1
    activation built, 2 done, 4 first stage ready, 5 first stage computed,
    6 first input pass, 7 rms scale known). One GPU: TinyLlama (config 1);
    under torchrun: Llama-3-8B tensor parallel over the ranks (config 4),
    every rank printing its own timeline."""
    import numpy as np
    from arm_ai_b200 import native, synth, tp
    if d.world > 1:
        arch = "llama-3-8b"
        if d.rank == 0:
            synth.model_path(arch, seed=0)
        d.barrier()
        uid = tp.share_unique_id(d.rank)
        m = tp.load_tp(synth.model_path(arch, seed=0), d.local, d.world, d.rank, uid, max_seq_len=1024)
    else:
        m = native.llama_candle_load_op(synth.model_path(ARCH, seed=0), max_seq_len=1024)
    native.llama_forward(m, synth.prompt_tokens(PROMPT, m.info().n_vocab, 3), 0, want_logits=False)
    for i in range(8):
        native.llama_forward(m, [5 + i], PROMPT + i, want_logits=False)
    for _ in range(2):
        tr = native.llama_trace_decode(m).astype(np.int64)
    m.close()
    out = []
    print_ = out.append
    nph, nct, _ = tr.shape
    t0 = tr[nph - 1, :, 0][tr[nph - 1, :, 0] > 0].min()
    names = ["QKV", "ATTN", "WO", "GATEUP", "DOWN"]
    nl = (nph - 2) // 5
    med = lambda a: float(np.median(a)) if len(a) else float("nan")
    end = {}
    rows = {}
    for i in range(nph - 1):
        ok = (tr[i, :, 0] > 0) & (tr[i, :, 2] > 0)
        if not ok.any():
            continue
        st, en = med(tr[i, ok, 0]) - t0, med(tr[i, ok, 2]) - t0
        a = ok & (tr[i, :, 1] > 0)
        act = med(tr[i, a, 1] - tr[i, a, 0]) if a.any() else 0.0
        end[i] = en
        kind = names[i % 5] if i < 5 * nl else "HEAD"
        rows.setdefault(kind, []).append((en - end.get(i - 1, 0.0), en - st, act))
    total = (tr[nph - 1, :, 1].max() - t0) / 1e3
    print_(f"decode step: {nph - 1} phases on {nct} CTAs, {total:.1f} us (trace build; globaltimer 256 ns resolution)")
    print_("| phase | n | span us (median) | own us | activation build us |")
    print_("|---|---|---|---|---|")
    for kind, v in rows.items():
        a = np.array(v) / 1e3
        print_(f"| {kind} | {len(v)} | {np.median(a[:, 0]):.2f} | {np.median(a[:, 1]):.2f} | {np.median(a[:, 2]):.2f} |")
    lm = nl // 2
    print_(f"layer {lm}, slot medians relative to the phase start (us; s3 = the producer issued the phase's "
           f"first weight chunk, s10 = consumers start waiting for it; polls = that wait's mbarrier polls):")
    for i in range(5 * lm, 5 * lm + 5):
        s0 = tr[i, :, 0]
        ok = s0 > 0
        cells = []
        for j in (3, 6, 7, 1, 10, 4, 5, 2):
            okj = ok & (tr[i, :, j] > 0)
            cells.append(f"s{j} {(med(tr[i, okj, j] - s0[okj])) / 1e3:.2f}" if okj.any() else f"s{j} -")
        okp = ok & (tr[i, :, 10] > 0)
        cells.append(f"polls {med(tr[i, okp, 11]):.0f}" if okp.any() else "polls -")
        print_(f"  {names[i % 5]:6s} " + "  ".join(cells))
    text = "\n".join(out)
    print((f"rank {d.rank} of {d.world}:\n" if d.world > 1 else "") + text, flush=True)


class Dist:
    def __init__(self):
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        self.pg = None
        if self.world > 1:
            import datetime

            import torch
            import torch.distributed as dist
            torch.cuda.set_device(self.local)
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                    device_id=torch.device("cuda", self.local))
            self.pg = dist

    def barrier(self):
        if self.pg:
            self.pg.barrier()

    def max(self, v: float) -> float:
        if not self.pg:
            return v
        import torch
        t = torch.tensor([v], dtype=torch.float64, device=f"cuda:{self.local}")
        self.pg.all_reduce(t, op=self.pg.ReduceOp.MAX)
        return float(t.item())

    def sum(self, v: float) -> float:
        if not self.pg:
            return v
        import torch
        t = torch.tensor([v], dtype=torch.float64, device=f"cuda:{self.local}")
        self.pg.all_reduce(t, op=self.pg.ReduceOp.SUM)
        return float(t.item())

    def close(self):
        if self.pg:
            self.pg.destroy_process_group()


class Clocks:
    """nvidia-smi samples (every 200 ms) during the timed region."""

    Q = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, dev: int, enabled: bool):
        self.dev, self.proc, self.lines = dev, None, []
        self.enabled = enabled

    def _smi_id(self):
        """nvidia-smi's id of CUDA device `dev`: its UUID, since nvidia-smi
        numbers GPUs in its own order and ignores CUDA_VISIBLE_DEVICES."""
        import torch
        return f"GPU-{torch.cuda.get_device_properties(self.dev).uuid}"

    def __enter__(self):
        if self.enabled:
            try:
                self.proc = subprocess.Popen(
                    ["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits", "-lms", "200",
                     "-i", self._smi_id()], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
                self.th = threading.Thread(target=self._read, daemon=True)
                self.th.start()
            except Exception:
                self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        if not self.lines:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 7:
                continue
            try:
                sm.append(float(f[0]))
                mx = float(f[1])
            except ValueError:
                continue
            for n, v in zip(names, f[3:7]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


def profiled_traffic(kernel):
    """DRAM bytes per launch of `kernel` from the committed ncu summary
    (profiles/<kernel>_tinyllama_b1.md, line "dram_bytes_per_launch = N")."""
    import re
    try:
        with open(os.path.join(ROOT, "profiles", f"{kernel}_tinyllama_b1.md")) as f:
            m = re.search(r"dram_bytes_per_launch = (\d+)", f.read())
        return int(m.group(1)) if m else None
    except OSError:
        return None


def measured_peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def cpu_model():
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def bench_config(world):
    """The `config` object of both arms' JSON lines (identical, so that the
    two lines describe the same workload)."""
    return {"workload": f"{ARCH} Q4_K_M greedy decode b=1: {PROMPT}-token prompt + {MAX_NEW} new "
                        f"tokens ({MAX_NEW - 1} timed decode steps per step)",
            "arch": "22 layers, hidden 2048, FFN 5632, 32/4 heads, head_dim 64, vocab 32000",
            "l2": "inputs larger than L2: every decode token streams all 633 MB of weights",
            "timed": "decode steps of one generation per step; prefill between steps untimed",
            "parallelism": f"replicas x{world}" if world > 1 else "1 GPU"}


def cpu_baseline_sample(path, prompt, max_new=6):
    """The oracle (candle's generic kernels restated in C, OpenMP over output
    columns as rayon does) on all host threads: decode tokens/s."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import ref
    cores = os.cpu_count() or 1
    ref.set_threads(cores)
    m = ref.OracleLlama(path)
    t0 = time.time()
    toks, pre_us, dec_us = m.generate(prompt, max_new)
    wall = time.time() - t0
    m.close()
    v = (len(toks) - 1) * 1e6 / max(dec_us, 1)
    return {"value": v, "unit": "tokens/s", "cores": cores, "kind": "port", "cpu": cpu_model(),
            "sample": f"{ARCH} Q4_K_M b=1: {len(prompt)}-token prompt + {max_new} new tokens "
                      f"(decode {len(toks) - 1} steps, {dec_us / 1e6:.1f} s; prefill {pre_us / 1e6:.1f} s; "
                      f"wall {wall:.1f} s)"}


def run_reference(args, d):
    """The reference's CPU path (the oracle restatement of candle 0.8.4's
    generic kernels, OpenMP over output columns as rayon does, all host
    threads) on the same workload as the GPU arm: per step one generation of
    a 32-token prompt + 128 new tokens, decode tokens/s measured as the
    reference measures it ((n_new - 1) / decode_us). Warm-up steps are
    shortened (8 new tokens): they only page the model in."""
    if d.rank != 0:
        return
    from arm_ai_b200 import synth
    path = synth.model_path(ARCH, seed=0)
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import ref
    cores = os.cpu_count() or 1
    ref.set_threads(cores)
    m = ref.OracleLlama(path)
    prompt = synth.prompt_tokens(PROMPT, m.n_vocab, 1000)
    for _ in range(args.warmup):
        m.generate(prompt, 8)
    tok, dec = 0, 0
    t0 = time.time()
    for _ in range(args.steps):
        toks, _, dec_us = m.generate(prompt, MAX_NEW)
        tok += len(toks) - 1
        dec += dec_us
    wall = time.time() - t0
    m.close()
    v = tok * 1e6 / max(dec, 1)
    out = {"metric": METRIC, "value": v, "unit": "tokens/s", "impl": "reference", "n_gpus": args.gpus,
           "steps": args.steps, "warmup": args.warmup, "ms_per_step": wall * 1000 / args.steps,
           "higher_is_better": True, "scaling": "weak", "vs_baseline": v / PUBLISHED_TOK_S, "dtype": "int8",
           "data": "synthetic (seeded random-init N(0,0.02) weights quantised Q4_K/Q6_K (Q4_K_M mix); "
                   "prompt ids uniform in [3, 32000))",
           "config": bench_config(args.gpus),
           "cpu_baseline": {"value": v, "unit": "tokens/s", "cores": cores, "kind": "port", "cpu": cpu_model(),
                            "sample": f"{args.steps} x ({PROMPT}-token prompt + {MAX_NEW} new tokens), "
                                      f"{tok} decode steps in {dec / 1e6:.1f} s"},
           "e2e": {"value": v, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(out), flush=True)


def run_config2(d):
    """Batched decode: 16 independent sequences, 512-token seeded prompts,
    128 new tokens each, sharded over the ranks (dp.generate_batch_dp); each
    rank decodes its sequences in one batched call. Reported beside the
    headline, measured after it."""
    from arm_ai_b200 import native, synth
    from arm_ai_b200.dp import generate_batch_dp, shard
    n_seq, plen, new = 16, 512, 128
    path = synth.model_path(ARCH, seed=0)
    local = len(shard(n_seq, d.world, d.rank))
    gpu = native.llama_candle_load_op(path, device=d.local, max_batch=max(local, 1), max_seq_len=1024,
                                      decode_kernel=1)
    prompts = [synth.prompt_tokens(plen, gpu.info().n_vocab, 2000 + i) for i in range(n_seq)]
    gen = lambda ps, mx, st: native.llama_generate_batch(gpu, ps, mx, st)
    generate_batch_dp(gen, prompts[: max(1, d.world)], 4)  # warm-up
    d.barrier()
    toks, pre_us, dec_us = generate_batch_dp(gen, prompts, new)
    gpu.close()
    n_dec = sum(len(t) - 1 for t in toks)
    return {"workload": f"{ARCH} Q4_K_M: {n_seq} sequences x ({plen}-token prompt + {new} new tokens), "
                        f"data-parallel over {d.world} GPU(s), batched decode per GPU",
            "decode_tokens_per_s": n_dec * 1e6 / max(dec_us, 1),
            "prefill_tokens_per_s": n_seq * plen * 1e6 / max(pre_us, 1),
            "decode_s": dec_us / 1e6, "prefill_s": pre_us / 1e6,
            "timing": "host wall clock around the batched call (max over ranks), as the reference times generate",
            "prefill_path": "tcgen05 GEMM (f16 operands, TMEM f32 accumulator), k_qgemm"}


def run_config4(d, peak):
    """Tensor-parallel decode: Llama-3-8B-architecture Q4_K_M, b = 1, 1024-token
    seeded prompt, 128 new tokens, tensor-parallel over the N ranks: decode
    by the persistent kernel, whose attn_output / ffn_down partial sums cross
    NVLink as generation-tagged peer-memory stores; prefill by the tensor-core
    GEMMs with NCCL all-reduces. Decode device-timed (CUDA events, max over
    ranks)."""
    from arm_ai_b200 import native, synth, tp
    arch = "llama-3-8b"
    if d.rank == 0:
        synth.model_path(arch, seed=0)
    d.barrier()
    path = synth.model_path(arch, seed=0)
    if d.world > 1:
        uid = tp.share_unique_id(d.rank)
        gpu = tp.load_tp(path, d.local, d.world, d.rank, uid, max_seq_len=2048)
    else:
        gpu = native.llama_candle_load_op(path, device=d.local, max_seq_len=2048)
    info = gpu.info()
    prompt = synth.prompt_tokens(1024, info.n_vocab, 3000)
    # warm-up at the timed length: first-use costs (NCCL buffers for this
    # message size, kernel variants of a 1024-token tile) stay out of the timing
    native.llama_forward(gpu, prompt, 0, want_logits=False)
    d.barrier()
    t0 = time.time()
    native.llama_forward(gpu, prompt, 0, want_logits=False)
    pre_s = d.max(time.time() - t0)
    n_dec = 127
    native.llama_bench_decode(gpu, 8)  # warm-up steps
    native.llama_forward(gpu, prompt, 0, want_logits=False)
    d.barrier()
    ms = d.max(native.llama_bench_decode(gpu, n_dec))
    step_s = ms / 1e3 / n_dec
    kv_row = 2 * info.n_layer * info.n_head_kv * info.head_dim * (2 if info.kv_f16 else 4)
    bytes_gpu = info.weight_bytes + kv_row * (1024 + 1024 + n_dec) / 2
    gpu.close()
    # batch 32: 32 independent 1024-token prompts, 128 new tokens each, one
    # batched greedy step per token (weights sharded the same way)
    try:
        b32 = run_config4_batch32(d, path, info, n_dec)
    except Exception as e:  # keep the b=1 figures; every rank takes this path
        b32 = {"error": repr(e)[:300]}
    return {"workload": f"{arch} Q4_K_M b=1: 1024-token prompt + {n_dec + 1} new tokens, "
                        f"{'tensor-parallel over ' + str(d.world) + ' GPUs (peer-memory partial sums)' if d.world > 1 else '1 GPU'}",
            "decode_tokens_per_s": 1.0 / step_s, "ms_per_token": step_s * 1e3,
            "prefill_tokens_per_s": 1024 / pre_s,
            "weight_stream_gb_s_per_gpu": bytes_gpu / step_s / 1e9,
            "frac_of_hbm_per_gpu": bytes_gpu / step_s / 1e9 / peak,
            "bytes_per_token_per_gpu": bytes_gpu,
            "timing": "decode: CUDA events over 127 back-to-back steps, max over ranks; prefill: host wall clock "
                      "(max over ranks), second 1024-token prefill",
            "batch32": b32}


def run_config4_batch32(d, path, info, n_dec):
    from arm_ai_b200 import native, synth, tp
    nb32 = 32
    if d.world > 1:
        uid = tp.share_unique_id(d.rank)
        gpu = tp.load_tp(path, d.local, d.world, d.rank, uid, max_seq_len=1024 + 160, max_batch=nb32)
    else:
        gpu = native.llama_candle_load_op(path, device=d.local, max_seq_len=1024 + 160, max_batch=nb32)
    prompts = [synth.prompt_tokens(1024, info.n_vocab, 3100 + s_) for s_ in range(nb32)]
    d.barrier()
    _, pre_us, dec_us = native.llama_generate_batch(gpu, prompts, n_dec + 1)
    dec32 = d.max(dec_us / 1e6)
    pre32 = d.max(pre_us / 1e6)
    gpu.close()
    return {"decode_tokens_per_s": nb32 * n_dec / dec32, "prefill_tokens_per_s": nb32 * 1024 / pre32,
            "decode_s": dec32, "prefill_s": pre32,
            "timing": "host wall clock around generate_batch's prefill and decode (max over ranks), "
                      "decode counted as (new tokens - 1) per sequence, as the reference counts it"}


def run_config3(d, peak):
    """Long-context decode: Mistral-7B-architecture Q4_K_M, b = 1, 4096-token
    seeded prompt with an f16 KV cache, then 256 decode tokens (split-K GQA
    attention over the long context). One GPU (rank 0 of a single-process
    run). Decode device-timed (CUDA events over 255 back-to-back steps)."""
    from arm_ai_b200 import native, synth
    arch, n_prompt, n_new = "mistral-7b", 4096, 256
    path = synth.model_path(arch, seed=0)
    gpu = native.llama_candle_load_op(path, device=d.local, max_seq_len=n_prompt + n_new + 64, kv_f16=1)
    info = gpu.info()
    prompt = synth.prompt_tokens(n_prompt, info.n_vocab, 4000)
    native.llama_forward(gpu, prompt, 0, want_logits=False)  # warm-up at the timed length
    t0 = time.time()
    native.llama_forward(gpu, prompt, 0, want_logits=False)
    pre_s = time.time() - t0
    n_dec = n_new - 1
    ms = native.llama_bench_decode(gpu, n_dec)
    step_s = ms / 1e3 / n_dec
    kv_row = 2 * info.n_layer * info.n_head_kv * info.head_dim * 2  # f16 K and V per position
    bytes_tok = info.weight_bytes + kv_row * (n_prompt + n_prompt + n_dec) / 2
    gpu.close()
    return {"workload": f"{arch} Q4_K_M b=1: {n_prompt}-token prompt (f16 KV) + {n_new} new tokens, 1 GPU",
            "decode_tokens_per_s": 1.0 / step_s, "ms_per_token": step_s * 1e3,
            "prefill_tokens_per_s": n_prompt / pre_s,
            "weight_and_kv_stream_gb_s": bytes_tok / step_s / 1e9,
            "frac_of_hbm": bytes_tok / step_s / 1e9 / peak,
            "bytes_per_token": bytes_tok,
            "timing": "decode: CUDA events over 255 back-to-back steps; prefill: host wall clock, second "
                      f"{n_prompt}-token prefill"}


def measured_tc_peak():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["bf16_tflops"]), "measured"
    except Exception:
        return 1590.0, "fallback"


def run_config5(d, peak_hbm):
    """BASELINE configs[4], the primitive sweep, through the device-pointer
    entry points (inputs resident in HBM): per call device time from CUDA
    events on the call's stream, L2 flushed (a 256 MB write) before every
    timed call, 3 warm-up calls, median of 10. Roofline per primitive: HBM
    for the matrix-vector shapes (int8 M <= 16, int4 matvecs, RMSNorm),
    tensor cores for the int8 GEMM at M = 512 (s8 dense peak taken as 2 x the
    measured bf16 GEMM peak, the nominal ratio) and for flash attention
    (measured bf16 peak)."""
    import ctypes

    import torch
    from arm_ai_b200._lib import load_cuda
    lib = load_cuda()
    dev = torch.device("cuda", d.local)
    torch.cuda.set_device(dev)
    st = torch.cuda.current_stream()
    sp = ctypes.c_void_p(st.cuda_stream)
    tc_peak, tc_src = measured_tc_peak()
    flush = torch.empty(64 * 1024 * 1024, dtype=torch.float32, device=dev)
    gen = torch.Generator(device=dev)
    gen.manual_seed(5)

    def timeit(fn):
        for _ in range(3):
            fn()
        times = []
        for _ in range(10):
            flush.fill_(1.0)
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(st)
            rc = fn()
            b.record(st)
            if rc != 0:
                raise RuntimeError(f"primitive call failed ({rc})")
            b.synchronize()
            times.append(a.elapsed_time(b))
        return statistics.median(times)

    P = lambda t: ctypes.c_void_p(t.data_ptr())
    out = {"timing": "device time per call (CUDA events on the call's stream), L2 flushed before each, median of 10",
           "tensor_peak_tflops": tc_peak, "tensor_peak_source": tc_src, "hbm_peak_gbs": peak_hbm}
    i8 = {}
    for K in (2048, 4096):
        w = torch.randint(-127, 128, (K, K), dtype=torch.int8, device=dev, generator=gen)
        ws = torch.rand(K, device=dev, generator=gen) * 0.1
        for M in (1, 16, 512):
            a = torch.randint(-127, 128, (M, K), dtype=torch.int8, device=dev, generator=gen)
            o = torch.empty(M, K, dtype=torch.float32, device=dev)
            ms = timeit(lambda: lib.armai_dev_int8_matmul_f32(P(a), P(w), None, 0, ctypes.c_float(0.0125), P(ws),
                                                              P(o), M, K, K, sp))
            ops, byt = 2 * M * K * K, K * K + M * K + 4 * K + 4 * M * K
            e = {"us": ms * 1e3, "tops": ops / ms / 1e9, "gb_s": byt / ms / 1e6}
            if M >= 64:
                e.update(bound="tensor", kernel="k_i8gemm (tcgen05 kind::i8)", frac=e["tops"] / (2 * tc_peak))
            else:
                e.update(bound="hbm", kernel="k_int8_gemm (dp4a)", frac=e["gb_s"] / peak_hbm)
            i8[f"M{M}_K{K}_N{K}"] = e
    out["int8_matmul_f32"] = i8
    i4 = {}
    for N, K in ((4096, 4096), (14336, 4096)):
        wp = torch.randint(0, 256, (N, K // 2), dtype=torch.uint8, device=dev, generator=gen)
        sc = torch.rand(N, K // 32, device=dev, generator=gen) * 0.01
        a = torch.rand(1, K, device=dev, generator=gen) * 2 - 1
        o = torch.empty(N, device=dev)
        byt = N * K // 2 + 4 * N * K // 32 + 4 * K + 4 * N
        for name, fn in (("int4_gemv_q4_x_q8", lambda: lib.armai_dev_int4_gemv_q4_x_q8(P(a), P(wp), P(sc), P(o), N,
                                                                                        K, sp)),
                         ("int4_matmul_f32_m1", lambda: lib.armai_dev_int4_matmul_f32(P(a), P(wp), P(sc), P(o), 1,
                                                                                        N, K, sp))):
            ms = timeit(fn)
            i4[f"{name}_N{N}_K{K}"] = {"us": ms * 1e3, "gb_s": byt / ms / 1e6, "bound": "hbm",
                                        "frac": byt / ms / 1e6 / peak_hbm}
    out["int4_matvec"] = i4
    x = torch.rand(512, 4096, device=dev, generator=gen)
    g = torch.rand(4096, device=dev, generator=gen)
    o = torch.empty_like(x)
    ms = timeit(lambda: lib.armai_dev_rmsnorm_f32(P(x), P(g), P(o), 512, 4096, ctypes.c_float(1e-5), sp))
    byt = 2 * 4 * 512 * 4096 + 4 * 4096
    out["rmsnorm_f32_512x4096"] = {"us": ms * 1e3, "gb_s": byt / ms / 1e6, "bound": "hbm",
                                   "frac": byt / ms / 1e6 / peak_hbm}
    H, S, D = 32, 2048, 128
    q, k, v = (torch.rand(1, H, S, D, device=dev, generator=gen).half() * 2 - 1 for _ in range(3))
    o = torch.empty(1, H, S, D, device=dev)
    ms = timeit(lambda: lib.armai_dev_flash_attention_f16(P(q), P(k), P(v), P(o), ctypes.c_float(D ** -0.5), 1, H,
                                                          S, S, D, 1, sp))
    fl = 4 * S * S * D * H / 2
    out["flash_attention_f16_h32_s2048_d128_causal"] = {"us": ms * 1e3, "tflops": fl / ms / 1e9, "bound": "tensor",
                                                        "frac": fl / ms / 1e9 / tc_peak,
                                                        "kernel": "k_fa_tc (tcgen05 kind::f16, P in tensor memory)"}
    return out


def run_armai(args, d):
    from arm_ai_b200 import native, synth
    if d.rank == 0:
        path = synth.model_path(ARCH, seed=0)
    d.barrier()
    path = synth.model_path(ARCH, seed=0)
    gpu = native.llama_candle_load_op(path, device=d.local)
    info = gpu.info()
    prompt = synth.prompt_tokens(PROMPT, info.n_vocab, 1000 + d.rank)
    n_dec = MAX_NEW - 1

    def decode_once():
        native.llama_forward(gpu, prompt, 0, want_logits=False)  # prefill (not timed)
        return native.llama_bench_decode(gpu, n_dec)

    for _ in range(args.warmup):
        decode_once()
    with Clocks(d.local, not args.no_clocks) as clk:
        d.barrier()
        t_wall = time.time()
        ms = [decode_once() for _ in range(args.steps)]
        t_wall = time.time() - t_wall
        d.barrier()
    dev_s = sum(ms) / 1e3
    max_s = d.max(dev_s)
    total_tokens = d.sum(args.steps * n_dec)
    value = total_tokens / max_s

    # e2e: through the C ABI generate call, host prompt in, every token out
    e2e_dec, e2e_tok, e2e_wall, pre_us_all = 0, 0, 0.0, 0
    for _ in range(max(1, args.steps)):
        t0 = time.time()
        toks, pre_us, dec_us = native.llama_candle_generate_op(gpu, prompt, MAX_NEW, [])
        e2e_wall += time.time() - t0
        e2e_dec += dec_us
        e2e_tok += len(toks) - 1
        pre_us_all += pre_us
    e2e_rank = e2e_tok * 1e6 / max(e2e_dec, 1)
    e2e_total = d.sum(e2e_rank)

    # Roofline of the dominant kernel. With the persistent decode kernel the
    # whole decode step is one launch: its algorithmic bytes are the step's
    # weight bytes plus the KV cache it reads (average context of the timed
    # generation), its duration the device time per step measured above.
    peak, peak_kind = measured_peaks()
    bytes_tok = info.weight_bytes
    kv_row = 2 * info.n_layer * info.n_head_kv * info.head_dim * (2 if info.kv_f16 else 4)
    kv_bytes = kv_row * (PROMPT + 1 + PROMPT + n_dec) / 2
    step_s = max_s / (args.steps * n_dec)
    ws_gbs = (bytes_tok + kv_bytes) / step_s / 1e9
    per_op = {}
    for kind in ("gateup", "ffn_down", "qkv", "attn_output", "head"):
        m_, b_ = native.llama_bench_kernel(gpu, kind, rounds=5)
        per_op[kind] = {"us": m_ * 1e3, "gb_s": b_ / (m_ * 1e-3) / 1e9}
    if info.n_kernels_per_step == 1:
        kname = "k_decode_mega"
        achieved = ws_gbs
        traffic = profiled_traffic(kname)
    else:
        kname = "k_matvec_gateup"
        ms_k, bytes_k = native.llama_bench_kernel(gpu, "gateup", rounds=5)
        achieved = bytes_k / (ms_k * 1e-3) / 1e9
        traffic = None
    gpu_launches = int(args.steps * n_dec * info.n_kernels_per_step * d.world)
    gpu.close()
    def guard(fn, *a):  # a failing side figure must not cost the headline line
        try:
            return fn(*a)
        except Exception as e:
            return {"error": repr(e)[:300]}
    cfg2 = None if args.no_config2 else guard(run_config2, d)
    cfg3 = guard(run_config3, d, peak) if (d.world == 1 and not args.no_config3) else None
    cfg4 = None if args.no_config4 else guard(run_config4, d, peak)
    cfg5 = guard(run_config5, d, peak) if (d.rank == 0 and not args.no_config5) else None
    cpu = None
    if d.rank == 0 and d.world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline_sample(path, prompt)
    if d.rank == 0:
        out = {
            "metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": d.world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": max_s * 1e3 / args.steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": value / d.world / PUBLISHED_TOK_S, "dtype": "int8",
            "data": "synthetic (seeded random-init N(0,0.02) weights quantised Q4_K/Q6_K (Q4_K_M mix); "
                    "prompt ids uniform in [3, 32000))",
            "config": bench_config(d.world),
            "weight_stream": {"gb_s_per_gpu": ws_gbs, "frac_of_hbm": ws_gbs / peak,
                              "bytes_per_token": bytes_tok + kv_bytes, "peak_gbs": peak, "peak_source": peak_kind},
            "decode_kernel": kname,
            "e2e": {"value": e2e_total, "unit": "tokens/s",
                    "h2d_bytes_per_step": PROMPT * 4, "d2h_bytes_per_step": MAX_NEW * 4,
                    "wall_tokens_per_s_incl_prefill": e2e_tok / max(e2e_wall, 1e-9) * d.world,
                    "prefill_tokens_per_s": PROMPT * 1e6 / max(pre_us_all / max(1, args.steps), 1)},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "traffic": traffic, "kernel": kname,
                         "algorithmic_bytes_per_launch": bytes_tok + kv_bytes,
                         "launch_us": step_s * 1e6, "peak_source": peak_kind,
                         "traffic_source": "profiles/k_decode_mega_tinyllama_b1.md (ncu dram__bytes_read.sum + "
                                           "dram__bytes_write.sum, one launch)" if traffic else None,
                         "per_op_kernels": per_op},
            "cpu_baseline": cpu,
            "clocks": clk.summary(),
            "gpu_launches": gpu_launches,
            "wall_s_timed_region": t_wall,
            "config2_batched": cfg2,
            "config3_mistral_7b_long": cfg3,
            "config4_llama3_8b": cfg4,
            "config5_primitives": cfg5,
        }
        print(json.dumps(out), flush=True)


def main():
    args = parse()
    if args.profile:
        _profile_case(args.profile)
        return
    d = Dist()
    if args.trace_decode:
        try:
            _trace_decode(d)
        finally:
            d.close()
        return
    try:
        if args.impl == "reference":
            run_reference(args, d)
        else:
            run_armai(args, d)
    finally:
        d.close()


if __name__ == "__main__":
    main()
