"""Headline benchmark: int4 Qwen3-8B decode tok/s on B200 (+ bs32 decode, prefill, qmatvec roofline).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]

Workload (BASELINE config 4 on one GPU): Qwen3-8B architecture (36 layers,
hidden 4096, 32 Q / 8 KV heads, head_dim 128, SwiGLU 12288, vocab 151936),
seeded N(0, 0.02) weights generated on the GPU and quantized by this repo's
sm_100a implementation of the reference quantizer: every linear Q4_K (int4,
32-value sub-blocks with 6-bit scales under fp16 super-block scales), LM head
Q6_K (the Q4_K_M head type), embeddings F16, norms F32.  A 1024-token random
prompt is prefilled, then one "step" = one greedy decode token per sequence,
replayed from a CUDA graph.  `value` = decode tokens/s over all ranks.

N > 1 (torchrun, one rank per GPU): tensor parallelism over the N ranks (heads,
rows and the vocabulary sharded; the row-parallel partial sums meet in a
peer-memory all-reduce), the same model and batch as N = 1, so `scaling` is
"strong".
"""

from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np
import torch

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))

PROMPT = 1024
BATCH_LARGE = 32
PEAKS_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}


def peaks() -> tuple[dict, str]:
    path = REPO / "MEASURED_PEAKS.json"
    if path.exists():
        return json.loads(path.read_text()), "measured"
    return PEAKS_FALLBACK, "fallback"


# ------------------------------------------------------------------ clocks
class ClockSampler:
    """nvidia-smi sampling of SM clocks and throttle reasons while running."""

    FIELDS = ("clocks.sm,clocks.max.sm,clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int) -> None:
        self.gpu = gpu_index
        self.proc: subprocess.Popen | None = None
        self.lines: list[str] = []
        self._thread: threading.Thread | None = None

    def __enter__(self) -> "ClockSampler":
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "200",
                 "-i", str(self.gpu)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self._thread = threading.Thread(target=self._read, daemon=True)
            self._thread.start()
            # nvidia-smi's own start-up (driver / NVML initialisation) must be over before the
            # timed region begins: wait for its first sample (at most 5 s)
            deadline = time.monotonic() + 5.0
            while not self.lines and time.monotonic() < deadline and self.proc.poll() is None:
                time.sleep(0.02)
            time.sleep(0.05)
        except FileNotFoundError:
            self.proc = None
        return self

    def _read(self) -> None:
        assert self.proc is not None and self.proc.stdout is not None
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc) -> None:
        if self.proc is not None:
            time.sleep(0.1)
            self.proc.terminate()
            self.proc.wait(timeout=5)
            if self._thread is not None:
                self._thread.join(timeout=2)

    def summary(self) -> dict:
        mhz, max_mhz, reasons = [], 0.0, set()
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        for line in self.lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) != 6:
                continue
            try:
                mhz.append(float(parts[0]))
                max_mhz = max(max_mhz, float(parts[1]))
            except ValueError:
                continue
            for name, flag in zip(names, parts[2:]):
                if flag.lower() == "active":
                    reasons.add(name)
        mhz.sort()
        return {"sm_mhz": mhz[len(mhz) // 2] if mhz else None, "sm_max_mhz": max_mhz or None,
                "reasons": sorted(reasons), "samples": len(mhz)}


# ---------------------------------------------------------------- helpers
def events_time(fn, reps: int, stream: torch.cuda.Stream) -> float:
    """Seconds per rep of fn() measured with CUDA events on `stream`."""
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    start.record(stream)
    for _ in range(reps):
        fn()
    end.record(stream)
    end.synchronize()
    return start.elapsed_time(end) * 1e-3 / reps


def dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch.distributed as dist

        torch.cuda.set_device(local)
        os.environ.setdefault("NCCL_DEBUG", "WARN")  # stdout carries only the JSON line
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    elif torch.cuda.is_available():
        torch.cuda.set_device(local)
    return world, rank, local


def barrier(world: int) -> None:
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def max_over_ranks(value: float, world: int) -> float:
    if world == 1:
        return value
    import torch.distributed as dist

    t = torch.tensor([value], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def traffic_from_profile() -> float | None:
    """DRAM bytes per launch of the dominant kernel from the committed ncu summary."""
    path = REPO / "profiles" / "qmv_swiglu_q4k_qwen3_8b.txt"
    if not path.exists():
        return None
    for line in path.read_text().splitlines():
        if line.startswith("traffic_bytes_per_launch:"):
            return float(line.split(":", 1)[1].strip())
    return None


# -------------------------------------------------------------- TP parity
def tp_parity(world: int, rank: int, local: int, steps: int = 32) -> dict:
    """Greedy tokens of the tensor-parallel runner against the single-GPU runner (rank 0 compares).

    A seeded 4-layer model with the 8B head layout (32 Q / 8 KV heads, 4096-wide projections, which
    split over 2, 4 and 8 ranks at super-block boundaries), Q4_K linears and a Q6_K head, 24-token prompt,
    `steps` graph-replayed decode steps on every rank.  The comparison against the CPU oracle runs in
    tests/test_tp_gpu.py; this line shows that the measured configuration decodes the same tokens.
    """
    import torch.distributed as dist

    from torch2vk_b200 import kernels
    from torch2vk_b200.qwen3 import Qwen3Config, Qwen3Runner, random_weights
    from torch2vk_b200.tp import make_tp_runner

    dev = torch.device("cuda", local)
    small = Qwen3Config(hidden=1024, layers=4, heads=32, kv_heads=8, head_dim=128, intermediate=4096, vocab=8192)
    w = random_weights(small, seed=1, device=str(dev), lm_head_kind="q6_k", topology="q4_k")
    ids = torch.randint(0, small.vocab, (1, 24), generator=torch.Generator().manual_seed(0)).to(dev)
    tp_runner = make_tp_runner(small, w, rank=rank, tp=world, batch=1, max_seq=96, max_new_tokens=steps + 2)
    got = tp_runner.generate(ids, steps).clone()
    torch.cuda.synchronize()
    everyone = [torch.empty_like(got) for _ in range(world)]
    dist.all_gather(everyone, got)
    result = {"steps": steps, "first_diff": None, "ranks_identical": all(torch.equal(e, got) for e in everyone),
              "reference": "single-GPU runner on the same weights"}
    if rank == 0:
        single = Qwen3Runner(small, w, batch=1, max_seq=96, max_new_tokens=steps + 2)
        ref = single.generate(ids, steps)
        ne = (ref.cpu() != got.cpu()).nonzero()
        result["first_diff"] = int(ne[0, -1]) if ne.numel() else steps
        single._graph = None
        del single
    result["device_status_bits"] = kernels.device_status()
    dist.barrier()
    tp_runner._graph = None
    if tp_runner._peer is not None:
        tp_runner._peer.close()
    del tp_runner
    torch.cuda.synchronize()
    return result


# ------------------------------------------------------------ CPU baseline
def cpu_baseline(sample_layers: int = 3, steps: int = 6) -> dict:
    """The reference PyTorch CPU path (HF fp32 Qwen3, dequantized-weight math) timed on the host cores.

    Bounded sample: HF Qwen3-8B-shaped models with 1 and `sample_layers`
    decoder layers (plus the full embedding / LM head) decode `steps` tokens
    each after a 32-token prompt; the median per-token times give the head
    cost and the per-layer cost, and the per-token time is that of 36 layers
    plus the head.  Weight values do not change the fp32 arithmetic cost, so
    the sample uses the HF default N(0, 0.02) init.
    """
    from oracle import qwen3_ref
    from transformers import Qwen3ForCausalLM

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)

    @torch.no_grad()
    def per_token(layers: int) -> float:
        torch.manual_seed(0)
        cfg = qwen3_ref.hf_config(4096, layers, 32, 8, 128, 12288, 151936)
        model = Qwen3ForCausalLM(cfg).float().eval()
        ids = qwen3_ref.prompt_ids(32, 151936, seed=0)
        out = model(input_ids=ids, use_cache=True)
        past, nxt = out.past_key_values, out.logits[:, -1:, :].argmax(-1)
        times = []
        for _ in range(steps + 1):
            t0 = time.perf_counter()
            out = model(input_ids=nxt, past_key_values=past, use_cache=True)
            past, nxt = out.past_key_values, out.logits[:, -1:, :].argmax(-1)
            times.append(time.perf_counter() - t0)
        times = sorted(times[1:])
        return times[len(times) // 2]

    t1 = per_token(1)
    tn = per_token(sample_layers)
    per_layer = max((tn - t1) / (sample_layers - 1), 0.0)
    head = max(t1 - per_layer, 0.0)
    token = head + 36 * per_layer
    return {"value": 1.0 / token, "unit": "tok/s", "cores": threads, "kind": "port",
            "sample": f"HF fp32 Qwen3-8B shapes with 1 and {sample_layers} layers + full head on CPU, median of "
                      f"{steps} decode tokens after a 32-token prompt; per-layer {per_layer * 1e3:.1f} ms x 36 + "
                      f"head {head * 1e3:.1f} ms"}


def run_reference(args, world: int, rank: int) -> None:
    if rank != 0:
        return
    base = cpu_baseline()
    line = {"impl": "reference", "metric": "qwen3_8b_int4_decode_tok_s_bs1", "value": base["value"], "unit": "tok/s",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "higher_is_better": True,
            "dtype": "f32", "data": "synthetic", "cpu_baseline": base,
            "e2e": {"value": base["value"], "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "config": {"workload": "Qwen3-8B decode bs1 (reference PyTorch fp32 CPU path)"}}
    print(json.dumps(line), flush=True)


# -------------------------------------------------------------------- main
def run_profile(args, local: int) -> None:
    """Workloads for ncu, bracketed by cudaProfilerStart/Stop (use --profile-from-start off).

    decode: the Qwen3-8B bs1 decode graph (Q4_K linears, Q6_K head), --steps replays.
    decode32: the same at batch 32 on a synthetic 1024-position KV cache.
    prefill: --steps prefills of the 1024-token prompt (batch 1).
    attnp:  the causal prefill attention of Qwen3-8B (32 Q / 8 KV heads, D 128) over a 2048-token prompt,
            batch 1 (attn_prefill_umma_kernel), --steps launches.
    lmhead: the Q6_K LM head (151936 x 4096, fused RMSNorm, argmax partials) at batch 1, --steps launches.
    attn:   the fused decode attention of Qwen3-8B (32 Q / 8 KV heads, D 128) at position 1040 over
            48 layers' KV caches in turn (288 MB, larger than L2), 8 splits per KV head (one
            thread-block cluster, as the decode runner uses), --steps launches.
    gemm:   the prefill gate/up + SwiGLU GEMM (Q4_K 2 x 12288 x 4096, 1024 tokens) over 4 layers'
            weights in turn (226 MB), --steps launches.
    gemm32: the same GEMM at 32 tokens (the batch-32 decode's gate/up: stacked 64 + 64-row tiles).
    asr:    --steps forwards of the Qwen3-ASR-0.6B audio tower over 3000 seeded mel frames (as the
            asr_encoder figure).
    asrdec: --steps text-decoder steps of the config-5 pipeline at batch 16 (Qwen3-0.6B shapes, Q4_K_M
            linears, Q6_K head), after its prefill (as the asr_e2e figure's decode phase).
    qmv:    the gate/up + SwiGLU matvec (Q4_K 2 x 12288 x 4096) over 4 layers' weights
            in turn (226 MB, larger than L2), --steps launches.
    """
    from torch2vk_b200 import kernels
    from torch2vk_b200.qwen3 import Qwen3Config, Qwen3Runner, random_weights

    cfg = Qwen3Config.qwen3_8b()
    dev = torch.device("cuda", local)
    cudart = torch.cuda.cudart()
    if args.profile in ("decode", "decode32", "prefill"):
        weights = random_weights(cfg, seed=0, device=str(dev), lm_head_kind="q6_k", topology="q4_k")
        batch = BATCH_LARGE if args.profile == "decode32" else 1
        runner = Qwen3Runner(cfg, weights, batch=batch, max_seq=PROMPT + args.steps + args.warmup + 64,
                             max_new_tokens=args.steps + args.warmup + 8)
        prompt = torch.randint(0, cfg.vocab, (batch, PROMPT), generator=torch.Generator().manual_seed(0)).to(dev)
        if args.profile == "prefill":
            runner.prefill(prompt)
            torch.cuda.synchronize()
            cudart.cudaProfilerStart()
            for _ in range(args.steps):
                runner.prefill(prompt)
            torch.cuda.synchronize()
            cudart.cudaProfilerStop()
            return
        if args.profile == "decode32":
            for kc, vc in zip(runner.k_cache, runner.v_cache):
                kc.normal_(0, 0.5)
                vc.normal_(0, 0.5)
            runner.positions.fill_(PROMPT)
        else:
            runner.prefill(prompt)
        runner.capture()
        for _ in range(args.warmup):
            runner.step()
        torch.cuda.synchronize()
        cudart.cudaProfilerStart()
        for _ in range(args.steps):
            runner.step()
        torch.cuda.synchronize()
        cudart.cudaProfilerStop()
    elif args.profile == "attn":
        B, NH, NK, D, S, L = 1, cfg.heads, cfg.kv_heads, cfg.head_dim, 1536, 48
        caches = [(torch.randn(B, S, NK, D, device=dev, dtype=torch.float16),
                   torch.randn(B, S, NK, D, device=dev, dtype=torch.float16)) for _ in range(L)]
        q = torch.randn(B, NH * D, device=dev, dtype=torch.float16)
        k = torch.randn(B, NK * D, device=dev, dtype=torch.float16)
        v = torch.randn(B, NK * D, device=dev, dtype=torch.float16)
        w = torch.ones(D, device=dev)
        from torch2vk_b200.qwen3 import inv_freq

        inv = inv_freq(cfg).to(dev)
        pos = torch.full((B,), 1040, device=dev, dtype=torch.int32)
        splits = 8
        ws = kernels.attn_decode_fused_workspace(B, NH, NK, D, splits, dev)
        out = torch.empty(B, NH * D, device=dev, dtype=torch.float16)

        def one(i: int) -> None:
            kc, vc = caches[i % L]
            kernels.attn_decode_fused(q, k, v, w, w, inv, kc, vc, pos, batch=B, n_heads=NH, n_kv=NK, head_dim=D,
                                      splits=splits, workspace=ws, out=out)

        for i in range(args.warmup):
            one(i)
        torch.cuda.synchronize()
        cudart.cudaProfilerStart()
        for i in range(args.steps):
            one(i)
        torch.cuda.synchronize()
        cudart.cudaProfilerStop()
    elif args.profile == "attnp":
        B, NH, NK, D, S = 1, cfg.heads, cfg.kv_heads, cfg.head_dim, 2048
        gen = torch.Generator(device=dev).manual_seed(0)
        q = torch.randn(B * S, NH * D, device=dev, generator=gen).half() / 11.3
        kc = torch.randn(B, S, NK, D, device=dev, generator=gen).half() / 11.3
        vc = torch.randn(B, S, NK, D, device=dev, generator=gen).half()
        pos = torch.zeros(B, device=dev, dtype=torch.int32)
        out = torch.empty_like(q)

        def one() -> None:
            kernels.attn_prefill(q, kc, vc, pos, batch=B, tokens=S, n_heads=NH, n_kv=NK, head_dim=D, out=out)

        for _ in range(args.warmup):
            one()
        torch.cuda.synchronize()
        cudart.cudaProfilerStart()
        for _ in range(args.steps):
            one()
        torch.cuda.synchronize()
        cudart.cudaProfilerStop()
    elif args.profile == "lmhead":
        gen = torch.Generator(device=dev).manual_seed(0)
        w = kernels.quantize(torch.randn(cfg.vocab, cfg.hidden, device=dev, generator=gen) * 0.02, "q6_k")
        nw = torch.ones(cfg.hidden, device=dev)
        x = torch.randn(1, cfg.hidden, device=dev, generator=gen).half()
        g = (cfg.vocab + 3) // 4
        ps = torch.empty(1, g, device=dev)
        pt = torch.empty(1, g, device=dev, dtype=torch.int32)

        def one() -> None:
            kernels.lm_head_argmax(x, w, "q6_k", cfg.hidden, norm_weight=nw, partial_scores=ps, partial_tokens=pt)

        for _ in range(args.warmup):
            one()
        torch.cuda.synchronize()
        cudart.cudaProfilerStart()
        for _ in range(args.steps):
            one()
        torch.cuda.synchronize()
        cudart.cudaProfilerStop()
    elif args.profile == "asrdec":
        from torch2vk_b200.asr import AsrEncoderConfig, random_params
        from torch2vk_b200.asr_pipeline import AsrPipeline

        acfg = AsrEncoderConfig.qwen3_asr_0_6b()
        tcfg = Qwen3Config.qwen3_0_6b()
        tw = random_weights(tcfg, seed=0, device=str(dev), lm_head_kind="q6_k", topology="q4_k_m")
        gen = torch.Generator().manual_seed(1)
        prefix = torch.randint(0, tcfg.vocab, (1, 9), generator=gen)
        suffix = torch.randint(0, tcfg.vocab, (1, 6), generator=gen)
        pipe = AsrPipeline(acfg, random_params(acfg, seed=0), tcfg, tw, batch=16, frames=3000, prefix=9, suffix=6,
                           max_new_tokens=64, device=dev)
        rng = np.random.default_rng(4)
        clips = pipe.upload([rng.standard_normal((acfg.num_mel_bins, 3000)).astype(np.float32) for _ in range(16)])
        ids = pipe.prompt(prefix, suffix, placeholder=151646)
        pipe.transcribe(clips, ids)  # graph capture
        pipe.encode(clips)
        pipe.runner.prefill(ids, inject=(pipe.audio_positions, pipe.features))
        for _ in range(args.warmup):
            pipe.runner.step()
        torch.cuda.synchronize()
        cudart.cudaProfilerStart()
        for _ in range(args.steps):
            pipe.runner.step()
        torch.cuda.synchronize()
        cudart.cudaProfilerStop()
    elif args.profile == "asr":
        from torch2vk_b200.asr import AsrEncoderConfig, AsrEncoderRunner, prepare_inputs, random_params

        acfg = AsrEncoderConfig.qwen3_asr_0_6b()
        mel = np.random.default_rng(4).standard_normal((acfg.num_mel_bins, 3000)).astype(np.float32)
        arun = AsrEncoderRunner(acfg, random_params(acfg, seed=0), device=dev)
        atens = arun.upload(prepare_inputs(mel, acfg))
        for _ in range(args.warmup):
            arun.forward(atens)
        torch.cuda.synchronize()
        cudart.cudaProfilerStart()
        for _ in range(args.steps):
            arun.forward(atens)
        torch.cuda.synchronize()
        cudart.cudaProfilerStop()
    elif args.profile in ("gemm", "gemm32"):
        gen = torch.Generator(device=dev).manual_seed(0)
        pairs = []
        for _ in range(4):
            g = kernels.quantize(torch.randn(cfg.intermediate, cfg.hidden, device=dev, generator=gen) * 0.02, "q4_k")
            u = kernels.quantize(torch.randn(cfg.intermediate, cfg.hidden, device=dev, generator=gen) * 0.02, "q4_k")
            pairs.append((g, u))
        tokens = PROMPT if args.profile == "gemm" else BATCH_LARGE
        x = torch.randn(tokens, cfg.hidden, device=dev, dtype=torch.float16)
        out = torch.empty(tokens, cfg.intermediate, device=dev, dtype=torch.float16)
        for i in range(args.warmup):
            g, u = pairs[i % 4]
            kernels.linear_swiglu(x, g, u, "q4_k", cfg.hidden, out=out)
        torch.cuda.synchronize()
        cudart.cudaProfilerStart()
        for i in range(args.steps):
            g, u = pairs[i % 4]
            kernels.linear_swiglu(x, g, u, "q4_k", cfg.hidden, out=out)
        torch.cuda.synchronize()
        cudart.cudaProfilerStop()
    else:
        gen = torch.Generator(device=dev).manual_seed(0)
        pairs = []
        for _ in range(4):
            g = kernels.quantize(torch.randn(cfg.intermediate, cfg.hidden, device=dev, generator=gen) * 0.02, "q4_k")
            u = kernels.quantize(torch.randn(cfg.intermediate, cfg.hidden, device=dev, generator=gen) * 0.02, "q4_k")
            pairs.append((g, u))
        x = torch.randn(1, cfg.hidden, device=dev, dtype=torch.float16)
        nw = torch.ones(cfg.hidden, device=dev)
        out = torch.empty(1, cfg.intermediate, device=dev, dtype=torch.float16)
        for i in range(args.warmup):
            g, u = pairs[i % 4]
            kernels.linear_swiglu(x, g, u, "q4_k", cfg.hidden, norm_weight=nw, out=out)
        torch.cuda.synchronize()
        cudart.cudaProfilerStart()
        for i in range(args.steps):
            g, u = pairs[i % 4]
            kernels.linear_swiglu(x, g, u, "q4_k", cfg.hidden, norm_weight=nw, out=out)
        torch.cuda.synchronize()
        cudart.cudaProfilerStop()
    if kernels.device_status() != 0:
        raise SystemExit("device status bit set")


def run_sweep(args, local: int) -> None:
    """The isolated quantized-linear sweep: N x K in {4096 x 4096, 12288 x 4096,
    4096 x 12288, 151936 x 4096}, M in {1, 4, 16, 64, 256, 2048}, Q4_K (int4, 32-value sub-blocks) and
    Q8_0 (int8, blocks of 32); weights N(0, 0.02) quantized by this repo's GPU quantizer, x N(0, 1) fp16.

    Each point: enough weight copies that one pass over them exceeds L2 (the copies are used in turn);
    `--steps` launches captured in one CUDA graph (no host launch cost in the figure), `--warmup`
    replays, then 5 replays timed with CUDA events on the launching stream.
    Prints one JSON line per point: us per launch, weight GB/s, % of the measured HBM copy
    bandwidth and TFLOP/s (the roofline that binds: HBM at small M, tensor at large M)."""
    from torch2vk_b200 import kernels

    pk, src = peaks()
    hbm = float(pk["hbm_gbs"])
    dev = torch.device("cuda", local)
    stream = torch.cuda.current_stream(dev)
    torch.manual_seed(0)
    for kind in ("q4_k", "q8_0"):
        for n, k in ((4096, 4096), (12288, 4096), (4096, 12288), (151936, 4096)):
            one = kernels.quantize(torch.randn(n, k, device=dev) * 0.02, kind)
            wbytes = one.numel() * one.element_size()
            copies = max(1, -(-256 * 2**20 // wbytes))  # > 2 x L2 per pass
            ws = [one] + [one.clone() for _ in range(copies - 1)]
            for m in (1, 4, 16, 64, 256, 2048):
                x = torch.randn(m, k, device=dev, dtype=torch.float16)
                out = torch.empty(m, n, device=dev, dtype=torch.float16)
                i = [0]

                def launch() -> None:
                    w = ws[i[0] % copies]
                    i[0] += 1
                    kernels.linear(x, w, kind, k, out=out)

                launch()  # first call outside the capture (one-time kernel attribute set-up)
                torch.cuda.synchronize()
                graph = torch.cuda.CUDAGraph()
                with torch.cuda.graph(graph):
                    for _ in range(args.steps):
                        launch()
                for _ in range(args.warmup):
                    graph.replay()
                t = events_time(graph.replay, 5, stream) / args.steps
                del graph
                flops = 2.0 * m * n * k
                print(json.dumps({"kind": kind, "N": n, "K": k, "M": m, "us": round(t * 1e6, 2),
                                  "weight_GBps": round(wbytes / t / 1e9, 1),
                                  "hbm_frac": round(wbytes / t / 1e9 / hbm, 3), "TFLOPs": round(flops / t / 1e12, 1),
                                  "copies": copies, "peak_source": src}), flush=True)
            del ws, one
            torch.cuda.empty_cache()
    if kernels.device_status() != 0:
        raise SystemExit("device status bit set")


def run_attention(args, local: int) -> None:
    """Attention alone: fp16 GQA with 32 Q / 8 KV heads, head_dim 128, Q/K/V
    N(0, 1) / sqrt(128).  (a) causal prefill of S in {512, 2048, 8192} tokens at batch 1 and 8
    (attn_prefill_tc_kernel), roofline = tensor (4 B NH D S (S + 1) / 2 flop); (b) decode of one query
    token against KV caches of {1k, 4k, 16k, 32k} positions at batch 1, 16 and 64, the decode path of
    the runner (attn_decode_fused: q / k norm + RoPE + the new position's cache write + split attention,
    the split count chosen as Qwen3Runner chooses it), roofline = HBM (K + V bytes read).  Each point:
    `--warmup` untimed launches, then `--steps` launches in one CUDA graph timed with events (decode:
    the caches of every point exceed L2 from 1k positions at batch 16; smaller points are L2-resident and
    marked).  One JSON line per point."""
    from torch2vk_b200 import kernels

    pk, src = peaks()
    hbm, tc = float(pk["hbm_gbs"]), float(pk["bf16_tflops"])
    dev = torch.device("cuda", local)
    stream = torch.cuda.current_stream(dev)
    NH, NK, D = 32, 8, 128
    g = torch.Generator(device=dev).manual_seed(3)
    scale = 1.0 / np.sqrt(D)

    def timed(launch) -> float:
        launch()
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for _ in range(args.steps):
                launch()
        for _ in range(args.warmup):
            graph.replay()
        t = events_time(graph.replay, 3, stream) / args.steps
        del graph
        return t

    for B in (1, 8):
        for S in (512, 2048, 8192):
            q = torch.randn(B, S, NH, D, device=dev, generator=g).mul_(scale).half()
            kc = torch.randn(B, S, NK, D, device=dev, generator=g).mul_(scale).half()
            vc = torch.randn(B, S, NK, D, device=dev, generator=g).mul_(scale).half()
            pos = torch.zeros(B, dtype=torch.int32, device=dev)
            out = torch.empty_like(q)
            t = timed(lambda: kernels.attn_prefill(q, kc, vc, pos, batch=B, tokens=S, n_heads=NH, n_kv=NK,
                                                   head_dim=D, out=out))
            flops = 4.0 * B * NH * D * S * (S + 1) / 2
            print(json.dumps({"mode": "prefill", "B": B, "S": S, "us": round(t * 1e6, 1),
                              "TFLOPs": round(flops / t / 1e12, 1), "tensor_frac": round(flops / t / 1e12 / tc, 3),
                              "peak_source": src}), flush=True)
            del q, kc, vc, out
    torch.cuda.empty_cache()
    qw = torch.ones(D, device=dev)
    kw = torch.ones(D, device=dev)
    inv = 1.0 / (1e6 ** (torch.arange(0, D, 2, device=dev, dtype=torch.float32) / D))
    for B in (1, 16, 64):
        for L in (1024, 4096, 16384, 32768):
            max_seq = L + 64
            kc = torch.randn(B, max_seq, NK, D, device=dev, generator=g).mul_(scale).half()
            vc = torch.randn(B, max_seq, NK, D, device=dev, generator=g).mul_(scale).half()
            qkv = torch.randn(B, (NH + 2 * NK) * D, device=dev, generator=g).half()
            qi, ki, vi = qkv[:, :NH * D], qkv[:, NH * D:(NH + NK) * D], qkv[:, (NH + NK) * D:]
            pos = torch.full((B,), L - 1, dtype=torch.int32, device=dev)
            if max_seq <= 16384:
                splits = max(1, min(8, max(1, 296 // (B * NK)), max_seq // 64))
            else:
                splits = max(1, min(32, max(1, 592 // (B * NK)), max_seq // 64))
            ws = kernels.attn_decode_fused_workspace(B, NH, NK, D, splits, dev)
            out = torch.empty(B, NH * D, dtype=torch.float16, device=dev)
            t = timed(lambda: kernels.attn_decode_fused(qi, ki, vi, qw, kw, inv, kc, vc, pos, batch=B, n_heads=NH,
                                                        n_kv=NK, head_dim=D, splits=splits, workspace=ws, out=out))
            kv_bytes = 2.0 * B * NK * L * D * 2
            print(json.dumps({"mode": "decode", "B": B, "L": L, "splits": splits, "us": round(t * 1e6, 1),
                              "GBps": round(kv_bytes / t / 1e9, 1), "hbm_frac": round(kv_bytes / t / 1e9 / hbm, 3),
                              "l2_resident": kv_bytes < 2 * 126e6, "peak_source": src}), flush=True)
            del kc, vc, qkv, ws, out
            torch.cuda.empty_cache()
    if kernels.device_status() != 0:
        raise SystemExit("device status bit set")


def asr_e2e_figures(dev: torch.device) -> dict:
    """BASELINE config 5 end to end: B clips of 3000 seeded N(0, 1) log-mel frames -> the Qwen3-ASR-0.6B
    audio tower (Q8_0) -> 390 audio rows injected into a 405-token prompt -> Qwen3-0.6B-shaped text
    decoder (Q4_K_M linears, Q6_K head) -> 64 greedy tokens per clip, at B = 1, 4, 16.  Seeded random
    weights (no checkpoint here).  Each B: one untimed run (graph capture), then one run timed per phase
    with CUDA events; inputs uploaded before the timed region."""
    from torch2vk_b200.asr import AsrEncoderConfig, random_params
    from torch2vk_b200.asr_pipeline import AsrPipeline
    from torch2vk_b200.qwen3 import Qwen3Config, random_weights

    acfg = AsrEncoderConfig.qwen3_asr_0_6b()
    aparams = random_params(acfg, seed=0)
    tcfg = Qwen3Config.qwen3_0_6b()
    tw = random_weights(tcfg, seed=0, device=str(dev), lm_head_kind="q6_k", topology="q4_k_m")
    rng = np.random.default_rng(4)
    gen = torch.Generator().manual_seed(1)
    prefix = torch.randint(0, tcfg.vocab, (1, 9), generator=gen)
    suffix = torch.randint(0, tcfg.vocab, (1, 6), generator=gen)
    points = []
    for batch in (1, 4, 16):
        pipe = AsrPipeline(acfg, aparams, tcfg, tw, batch=batch, frames=3000, prefix=9, suffix=6, max_new_tokens=64,
                           device=dev)
        clips = pipe.upload([rng.standard_normal((acfg.num_mel_bins, 3000)).astype(np.float32) for _ in range(batch)])
        ids = pipe.prompt(prefix, suffix, placeholder=151646)
        pipe.transcribe(clips, ids)
        t = pipe.timed_transcribe(clips, ids)
        total = t.encoder_s + t.prefill_s + t.decode_s
        points.append({"batch": batch, "tok_s": batch * 64 / total, "encoder_ms": t.encoder_s * 1e3,
                       "prefill_ms": t.prefill_s * 1e3, "decode_ms": t.decode_s * 1e3,
                       "prompt_tokens": pipe.prompt_len})
        pipe.runner._graph = None
        del pipe, clips
        torch.cuda.empty_cache()
    del tw
    return {"workload": "Qwen3-ASR-0.6B-shaped: 3000-frame clips, audio tower + 28-layer text decoder, 64 greedy "
                        "tokens per clip (seeded weights)", "points": points}


def omnivoice_figures(dev: torch.device, stream: torch.cuda.Stream) -> dict:
    """OmniVoice's LLM forward, the per-step program of its 32-step masked iterative decoding: the CFG pair
    (batch 2) over the reference export's 85 positions (14 style + 21 text ids + 50 target audio positions),
    Qwen3-0.6B-shaped LLM (28 layers, Q4_K_M), Q8_0 text / audio embeddings, Q6_K audio heads (8 x 1025),
    seeded weights; one graph-replayed step timed over 20 replays, and the 32 steps of one utterance
    (the CFG scoring and token update between steps are not part of this path)."""
    from torch2vk_b200.omnivoice import OmniVoiceConfig, OmniVoiceLLM, prepare_inputs, random_weights

    cfg = OmniVoiceConfig.omnivoice()
    w = random_weights(cfg, seed=0, device=str(dev))
    rng = np.random.default_rng(5)
    inputs = prepare_inputs(rng.integers(0, cfg.llm.vocab, 14), rng.integers(0, cfg.llm.vocab, 21), 50, cfg)
    llm = OmniVoiceLLM(cfg, w, batch=2, seq=inputs.input_ids.shape[2])
    llm.forward(inputs)
    for _ in range(3):
        llm.forward()
    t = events_time(llm.forward, 20, stream)
    tokens = 2 * inputs.input_ids.shape[2]
    llm._graph = None
    del llm, w
    torch.cuda.empty_cache()
    return {"workload": "OmniVoice LLM forward (CFG pair, 85 positions, 28 layers, audio heads), seeded weights",
            "step_ms": t * 1e3, "tokens_per_step": tokens, "tok_s": tokens / t, "utterance_32_steps_ms": 32 * t * 1e3}


def qwen3_0_6b_figures(dev: torch.device, stream: torch.cuda.Stream) -> dict:
    """BASELINE config 1 on the fused runner: Qwen3-0.6B architecture (28 layers, hidden 1024, 16 Q / 8 KV
    heads, FFN 3072, vocab 151936, tied-embedding shapes), seeded weights quantized on the GPU (Q4_K
    linears, Q6_K head, F16 embedding), batch 1: a 128-token random prompt prefilled, then 128 greedy decode
    steps replayed from the CUDA graph."""
    from torch2vk_b200.qwen3 import Qwen3Config, Qwen3Runner, random_weights

    cfg = Qwen3Config.qwen3_0_6b()
    w = random_weights(cfg, seed=0, device=str(dev), lm_head_kind="q6_k", topology="q4_k")
    runner = Qwen3Runner(cfg, w, batch=1, max_seq=128 + 128 + 16, max_new_tokens=128 + 8)
    prompt = torch.randint(0, cfg.vocab, (1, 128), generator=torch.Generator().manual_seed(0)).to(dev)
    runner.prefill(prompt)
    t_pre = events_time(lambda: runner.prefill(prompt), 3, stream)
    runner.prefill(prompt)
    runner.capture()
    runner.step()  # the captured step's first replay
    t_dec = events_time(runner.step, 127, stream)
    runner._graph = None
    del runner, w
    torch.cuda.empty_cache()
    return {"workload": "Qwen3-0.6B, batch 1, 128-token prompt then 128 greedy decode steps (CUDA-graph replay)",
            "prefill_tok_s": 128 / t_pre, "decode_tok_s": 1.0 / t_dec}


def run_session(args, local: int) -> None:
    """The bs1 decode step of a Qwen3-0.6B-shaped model dispatched through RuntimeSession, the
    reference-facing path (286 dispatches a step): `--warmup` direct frames, then a replay plan of the
    last one, captured into a CUDA graph on its first execution and stepped `--steps` times with the
    step's input staged from the host and the next token read back every step.  One JSON line."""
    import tempfile

    from torch2vk_b200.qwen3_session import SessionDecodeModel
    from torch2vk_b200.runtime.replay import execute_replay, stage_replay_step_inputs
    from torch2vk_b200.runtime.session import RuntimeSession

    torch.cuda.set_device(local)
    m = SessionDecodeModel()
    d = Path(tempfile.mkdtemp())
    m.write_gguf(d)
    x = (np.random.default_rng(0).standard_normal((1, 1, m.hidden)) * 0.5).astype(np.float16)
    eos = np.array([151643, 151645], np.int64)
    start = 128
    with RuntimeSession.open(model_dir=d, model_tensors=m.weights) as rt:
        rt.materialize_model_weights()
        with rt.request(state=m.request_state()):
            direct = []
            for j in range(args.warmup):
                torch.cuda.synchronize()
                t0 = time.perf_counter()
                with rt.frame(f"decode.{j}"):
                    rt.register_host_inputs({m.x_in: x, m.eos: eos})
                    m.step(rt, start + j, j)
                    rt.readback(m.next_token)
                direct.append((time.perf_counter() - t0) * 1e3)
            plan = rt.build_replay_plan(name="decode", frame=f"decode.{args.warmup - 1}",
                                        readback_tensors={"next": m.next_token})

            def run(j: int) -> None:
                stage_replay_step_inputs(rt, plan=plan, inputs={m.x_in: x, m.eos: eos})
                execute_replay(plan, dynamic_push_constants={"cache_position": start + j, "start_position": start + j,
                                                             "theta": 1e6, "token_index": j})

            j = args.warmup
            for _ in range(3):  # direct execution + capture, then two replays
                run(j)
                j += 1
            steps = max(1, min(args.steps, 511 - j))
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            for _ in range(steps):
                run(j)
                j += 1
            step_ms = (time.perf_counter() - t0) * 1e3 / steps
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            with torch.cuda.stream(rt.stream):
                e0.record()
                for _ in range(50):
                    plan.graph.replay()
                e1.record()
            torch.cuda.synchronize()
            graph_ms = e0.elapsed_time(e1) / 50
    print(json.dumps({"metric": "session_decode_tok_s", "value": round(1e3 / step_ms, 1), "unit": "tok/s",
                      "steps": steps, "warmup": args.warmup, "ms_per_step": round(step_ms, 4),
                      "graph_device_ms": round(graph_ms, 4), "direct_frame_ms": round(float(np.median(direct)), 3),
                      "dispatches": plan.num_dispatches, "graph_replays": plan.graph_replays,
                      "direct_executions": plan.direct_executions, "dtype": "fp16 x Q4_K / Q6_K", "data": "synthetic",
                      "config": {"workload": "Qwen3-0.6B-shaped bs1 decode through RuntimeSession "
                                             "(optimized variants, replay plan with device push constants)"}}))


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=400)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--profile", choices=["decode", "decode32", "prefill", "qmv", "attn", "attnp", "lmhead", "gemm",
                                          "gemm32", "asr", "asrdec"],
                    default=None,
                    help="profiling workload only (no JSON): the profiler range opens after warm-up")
    ap.add_argument("--sweep", action="store_true",
                    help="the quantized-linear sweep (one JSON line per shape, M and type) instead of the step")
    ap.add_argument("--attention", action="store_true",
                    help="time attention alone (BASELINE config 3 grid); one JSON line per point")
    ap.add_argument("--session", action="store_true",
                    help="the decode step through RuntimeSession and a replay plan (one JSON line) instead")
    args = ap.parse_args()
    if args.warmup < 3:
        raise SystemExit("--warmup must be >= 3")
    world, rank, local = dist_setup()
    if args.impl == "reference":
        run_reference(args, world, rank)
        return
    if args.profile:
        run_profile(args, local)
        return
    if args.sweep:
        run_sweep(args, local)
        return
    if args.session:
        run_session(args, local)
        return
    if args.attention:
        run_attention(args, local)
        return

    from torch2vk_b200 import kernels
    from torch2vk_b200.qwen3 import Qwen3Config, Qwen3Runner, random_weights, weight_bytes

    cfg = Qwen3Config.qwen3_8b()
    dev = torch.device("cuda", local)
    # N > 1: tensor parallelism over the N ranks (same seeded weights everywhere, each rank keeps its shard)
    full_weights = random_weights(cfg, seed=0, device=str(dev), lm_head_kind="q6_k", topology="q4_k")
    torch.cuda.synchronize()
    steps, warm = args.steps, args.warmup
    # every decode step a runner takes (warm-up, timed, e2e warm-up and e2e) gets its own
    # cache row and token slot: a step past the cache would be rejected by the kernels
    e2e_reps = min(steps, 200)
    decode_steps = warm + steps + 3 + e2e_reps
    stream = torch.cuda.current_stream(dev)
    if world > 1:
        import torch.distributed as dist

        from torch2vk_b200.tp import local_config, make_tp_runner, shard_weights

        warm_t = torch.ones(1, device=dev)
        dist.all_reduce(warm_t)  # NCCL communicator up before any graph capture
        kcfg = local_config(cfg, world)
        weights = shard_weights(full_weights, cfg, rank, world)

        def new_runner(batch: int):
            return make_tp_runner(cfg, full_weights, rank=rank, tp=world, batch=batch,
                                  max_seq=PROMPT + decode_steps + 64, max_new_tokens=decode_steps + 8)
    else:
        kcfg, weights = cfg, full_weights

        def new_runner(batch: int):
            return Qwen3Runner(cfg, weights, batch=batch, max_seq=PROMPT + decode_steps + 64,
                               max_new_tokens=decode_steps + 8)
    wb = weight_bytes(weights)
    parity = tp_parity(world, rank, local) if world > 1 else None

    # ---- prefill (1024-token prompt), timed with events
    runner = new_runner(1)
    gen = torch.Generator().manual_seed(0)
    prompt = torch.randint(0, cfg.vocab, (1, PROMPT), generator=gen).to(dev)
    runner.prefill(prompt)  # warm-up of every prefill launch path
    t_prefill = max_over_ranks(events_time(lambda: runner.prefill(prompt), 1, stream), world)
    runner.capture()

    # ---- bs1 decode: W warm-up replays, then K timed replays.  Every rank starts its clock sampler
    # first (its start-up takes up to seconds), then all ranks meet, so that the timed replays begin
    # together and no rank's first peer all-reduce waits on another rank's sampler start-up.
    for _ in range(warm):
        runner.step()
    with ClockSampler(local) as clocks:
        barrier(world)
        torch.cuda.synchronize()
        t_step = events_time(runner.step, steps, stream)
    barrier(world)
    t_step = max_over_ranks(t_step, world)
    status = kernels.device_status()

    # ---- e2e: host token in (pinned H2D), graph step, host token out (D2H), every step
    host_in = torch.zeros(1, dtype=torch.int64).pin_memory()
    host_out = torch.zeros(1, dtype=torch.int64).pin_memory()
    host_out.copy_(runner.next_token.cpu())

    def e2e_step() -> None:
        host_in.copy_(host_out)
        runner.next_token.copy_(host_in, non_blocking=True)
        runner.step()
        host_out.copy_(runner.next_token, non_blocking=True)
        stream.synchronize()

    for _ in range(3):
        e2e_step()
    t0 = time.perf_counter()
    for _ in range(e2e_reps):
        e2e_step()
    t_e2e = max_over_ranks((time.perf_counter() - t0) / e2e_reps, world)
    status |= kernels.device_status()

    # ---- dominant kernel: gate/up + SwiGLU matvec (Q4_K 2 x 12288 x 4096), all 36 layers' weights in turn
    x = torch.randn(1, kcfg.hidden, device=dev, dtype=torch.float16)
    act = torch.empty(1, kcfg.intermediate, device=dev, dtype=torch.float16)

    def swiglu_all() -> None:
        for lw in weights.layers:
            kernels.linear_swiglu(x, lw.gate.data, lw.up.data, "q4_k", kcfg.hidden, norm_weight=lw.post_norm,
                                  out=act)

    swiglu_all()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        swiglu_all()
    for _ in range(3):
        g.replay()
    t_kernel = events_time(g.replay, 10, stream) / cfg.layers
    kbytes = (weights.layers[0].gate.data.numel() * 4 * 2) + 2 * kcfg.hidden + 2 * kcfg.intermediate
    pk, pk_kind = peaks()

    # ---- bs32 decode on a synthetic 1024-position KV cache (same kernels, M = 32)
    runner._graph = None
    del runner
    torch.cuda.empty_cache()
    big = new_runner(BATCH_LARGE)
    for kc, vc in zip(big.k_cache, big.v_cache):
        kc.normal_(0, 0.5)
        vc.normal_(0, 0.5)
    big.positions.fill_(PROMPT)
    big.next_token.random_(0, cfg.vocab)
    big.capture()
    for _ in range(warm):
        big.step()
    reps32 = max(8, steps // 8)
    t_step32 = max_over_ranks(events_time(big.step, reps32, stream), world)

    per_step_launches = cfg.layers * (5 if big.fused_attention else 6 + (1 if big.decode_splits > 1 else 0)) + 5
    big._graph = None
    del big
    torch.cuda.empty_cache()

    # ---- ASR audio encoder (configuration 5: the Qwen3-ASR-0.6B audio tower, Q8_0 weights, 3000 seeded
    # synthetic mel frames -> 30 chunks -> 390 tokens); replicas only: every rank runs its own
    from torch2vk_b200.asr import AsrEncoderConfig, AsrEncoderRunner, prepare_inputs, random_params

    acfg = AsrEncoderConfig.qwen3_asr_0_6b()
    ainp = prepare_inputs(np.random.default_rng(4).standard_normal((acfg.num_mel_bins, 3000)).astype(np.float32), acfg)
    arun = AsrEncoderRunner(acfg, random_params(acfg, seed=0), device=dev)
    atens = arun.upload(ainp)
    for _ in range(3):
        arun.forward(atens)
    t_asr = max_over_ranks(events_time(lambda: arun.forward(atens), 5, stream), world)
    asr = {"workload": "Qwen3-ASR-0.6B audio encoder, 3000 mel frames (30 chunks, 390 tokens), Q8_0 weights",
           "ms": t_asr * 1e3, "tflops": arun.flops(ainp) / t_asr / 1e12}
    del arun, atens
    small = qwen3_0_6b_figures(dev, stream) if world == 1 else None
    asr_e2e = asr_e2e_figures(dev) if world == 1 else None
    omni = omnivoice_figures(dev, stream) if world == 1 else None
    clk = clocks.summary()
    line = {
        "metric": "qwen3_8b_int4_decode_tok_s_bs1",
        "value": 1.0 / t_step,
        "unit": "tok/s",
        "n_gpus": world,
        "steps": steps,
        "warmup": warm,
        "ms_per_step": t_step * 1e3,
        "higher_is_better": True,
        "scaling": "strong" if world > 1 else "weak",
        "vs_baseline": None,
        "dtype": "fp16 activations x Q4_K / Q6_K codes as exact fp16 (mma.sync f16, f32 accumulate)",
        "data": "synthetic (seeded random weights, random prompt ids)",
        "config": {"workload": "Qwen3-8B decode, batch 1, 1024-token prompt, Q4_K linears + Q6_K head",
                   "model": "qwen3-8b-arch", "global_batch": 1, "seq_len": PROMPT,
                   "parallelism": f"tp{world}" if world > 1 else "single GPU",
                   "l2": "weights (4.3 GB / tp per GPU) larger than L2 every step"},
        "e2e": {"value": 1.0 / t_e2e, "unit": "tok/s", "h2d_bytes_per_step": 8, "d2h_bytes_per_step": 8},
        "gpu_launches": per_step_launches * steps,
        "clocks": {"sm_mhz": clk["sm_mhz"], "sm_max_mhz": clk["sm_max_mhz"], "reasons": clk["reasons"]},
        "roofline": {
            "bound": "hbm",
            "kernel": "qmv_m1_kernel (gate/up + SwiGLU, Q4_K 2 x 12288 x 4096 per GPU / tp)",
            "achieved": kbytes / t_kernel / 1e9,
            "peak": pk["hbm_gbs"],
            "unit": "GB/s",
            "frac": kbytes / t_kernel / 1e9 / pk["hbm_gbs"],
            "peak_source": pk_kind,
            "traffic": traffic_from_profile(),
            "algorithmic_bytes_per_launch": kbytes,
        },
        "step_roofline": {
            "bytes_per_step": wb["linears"] + wb["lm_head"],
            "achieved_gbs": (wb["linears"] + wb["lm_head"]) / t_step / 1e9,
            "frac": (wb["linears"] + wb["lm_head"]) / t_step / 1e9 / pk["hbm_gbs"],
        },
        "decode_bs32_tok_s": BATCH_LARGE / t_step32,
        "prefill_tok_s": PROMPT / t_prefill,
        "asr_encoder": asr,
        "device_status_bits": status,
    }
    if parity is not None:
        line["tp_parity"] = parity
    if small is not None:
        line["qwen3_0_6b"] = small
    if asr_e2e is not None:
        line["asr_e2e"] = asr_e2e
    if omni is not None:
        line["omnivoice_llm"] = omni
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline()
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        import torch.distributed as dist

        # the decode graphs (which hold NCCL work) were released before the ASR section
        torch.cuda.synchronize()
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
