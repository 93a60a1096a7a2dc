#!/usr/bin/env python
"""Benchmark: Q4_K_M bs=1 decode tok/s + matvec HBM GB/s vs B200 peak.

Workload: Qwen3-0.6B-shaped decoder, Q4_K_M weights
N(0, 0.02) from seed 0 (synthetic: no model files exist on these machines), a
512-token uniform-random prompt (seed 1 + rank), 256 greedy tokens.  One
"step" is the decode of those 256 tokens after the prompt (positions
512..767); the prompt is prefilled once during setup.

  value   decode tok/s over all ranks, device-timed with CUDA events on the
          engine's stream, inputs resident in HBM
  e2e     the same decode through generateLlamaWgsl (the public API): host
          token in, 256 ids back to the host, wall-clock
  roofline  bytes the step must read (weights + KV) per token / average
          per-token kernel time, against MEASURED_PEAKS.json hbm_gbs
  cpu_baseline  the CPU oracle (a C restatement of the reference's WGSL
          kernels; the WebGPU runtime itself cannot run here) on a bounded
          sample of the same model, all host cores

Multi-GPU: independent replicas, one sequence per GPU, no collective on the
data path (scaling "weak").  `--impl reference` times the CPU restatement of
the reference on rank 0 only.
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
sys.path.insert(0, ROOT)

CONFIGS = {
    # name: (synth spec, prompt tokens, generated tokens, sampling)
    "qwen3-0.6b-q4_k_m": ("qwen3-0.6b", 512, 256, None),
    "smollm2-135m-q4_k_m": ("smollm2-135m", 32, 128, None),
    "qwen3-0.6b-q8_0": ("qwen3-0.6b-q8", 1920, 128, None),
    "gemma3-270m-q4_k_m": ("gemma3-270m", 64, 256, {"temperature": 1.0, "topK": 64, "topP": 0.95, "seed": 0}),
}
MAX_CONTEXT = {"qwen3-0.6b": 2048, "qwen3-0.6b-q8": 2048, "smollm2-135m": 512, "gemma3-270m": 512}
METRIC = "Q4_K_M bs=1 decode tok/s + matvec HBM GB/s vs B200 peak"
# 256 independent sequences, 128-token prompt + 256 greedy
# tokens each, continuous batching over a paged fp16 KV cache, sequences
# sharded across the GPUs (sequence i on rank i mod N), no collective.
BATCHED = {"spec": "smollm2-135m", "seqs": 256, "prompt": 128, "generated": 256, "max_context": 512}
BATCHED_METRIC = "batched decode aggregate tok/s (256 sequences, continuous batching)"


def log(*a):
    print(*a, file=sys.stderr, flush=True)


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def model_file(spec_name: str, rank: int, world: int, barrier, tokenizer: bool = False) -> str:
    import dataclasses
    from chonklm_b200.synth import SPECS, write_synthetic_gguf
    d = os.environ.get("CK_BENCH_DIR", "/tmp/chonk_bench_cpuq")
    os.makedirs(d, exist_ok=True)
    path = os.path.join(d, f"{spec_name}{'-tok' if tokenizer else ''}.gguf")
    if rank == 0 and not os.path.exists(path):
        t = time.time()
        spec = dataclasses.replace(SPECS[spec_name], tokenizer=True) if tokenizer else SPECS[spec_name]
        # quantized on the CPU: the same bytes on every machine, the bytes the
        # oracle fixture (tests/golden/bench_decode_ids.json) was made from
        write_synthetic_gguf(spec, path + ".tmp", seed=0, device="cpu")
        os.replace(path + ".tmp", path)
        log(f"[bench] wrote {path} in {time.time() - t:.1f}s")
    barrier()
    return path


class Clocks:
    """nvidia-smi samples during the timed region."""

    def __init__(self, index: int):
        self.index = index
        self.rows = []
        self.proc = None

    def __enter__(self):
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={q}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thr = threading.Thread(target=self._read, daemon=True)
            self.thr.start()
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.rows.append([c.strip() for c in line.split(",")])

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
        sm = [float(r[1]) for r in self.rows if len(r) > 2 and r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in self.rows if len(r) > 2 and r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = set()
        for r in self.rows:
            for i, n in enumerate(names):
                if len(r) > 5 + i and r[5 + i].lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": sorted(reasons), "samples": len(self.rows)}


def oracle_at_position(path: str, vocab: int, max_context: int, pos: int):
    """The oracle on the bench's model, its engine moved to position `pos`
    (the GPU arm's first decode position).  The prompt's KV rows are not
    computed: decoding at `pos` costs the same arithmetic whatever the cache
    holds (every position up to `pos` is attended), which is what the timing
    needs."""
    from oracle import oracle
    m = oracle.OracleModel(path, vocab=vocab, max_context=max_context)
    m.set_position(pos)
    return m


def cpu_baseline_sample(path: str, vocab: int, max_context: int, pos: int, seconds: float = 12.0):
    """Oracle (fp32, WGSL operation order, OpenMP over output rows) decode
    tok/s on the host cores: a bounded sample of the same model at the GPU
    arm's positions."""
    cores = os.cpu_count() or 1
    os.environ.setdefault("OMP_NUM_THREADS", str(cores))
    cores = int(os.environ["OMP_NUM_THREADS"])
    import numpy as np
    m = oracle_at_position(path, vocab, max_context, pos)
    nid = int(np.random.default_rng(1).integers(0, vocab))
    nid = m.run_token(nid, True)       # warm-up step (page-in of the weights)
    n = 0
    t0 = time.perf_counter()
    while n < 64:
        nid = m.run_token(nid, True)
        n += 1
        if time.perf_counter() - t0 > seconds:
            break
    dt = time.perf_counter() - t0
    m.close()
    return {"value": n / dt, "unit": "tok/s", "cores": cores, "kind": "port",
            "sample": f"{n} greedy decode steps of the same synthetic model at positions {pos + 1}..{pos + n} "
                      f"(the GPU arm decodes from {pos}; C oracle, fp32, OpenMP over rows, {cores} threads)"}


def run_reference(args, cfg_name, rank, world, barrier):
    if rank != 0:
        return
    spec, prompt_len, gen, sampling = CONFIGS[cfg_name]
    from chonklm_b200.synth import SPECS
    path = model_file(spec, 0, 1, lambda: None)
    vocab = SPECS[spec].vocab
    cores = os.cpu_count() or 1
    os.environ.setdefault("OMP_NUM_THREADS", str(cores))
    cores = int(os.environ["OMP_NUM_THREADS"])
    import numpy as np
    m = oracle_at_position(path, vocab, MAX_CONTEXT[spec], prompt_len)
    nid = int(np.random.default_rng(1).integers(0, vocab))
    per_step = 2   # tokens decoded per step: a bounded sample of the 256-token step
    for _ in range(args.warmup):
        for _ in range(per_step):
            nid = m.run_token(nid, True)
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        for _ in range(per_step):
            nid = m.run_token(nid, True)
        times.append(time.perf_counter() - t0)
    tot = sum(times)
    value = per_step * args.steps / tot
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000 * tot / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": cfg_name, "prompt": prompt_len, "generated": gen,
                       "note": "reference WebGPU runtime unavailable on this box (no Node/Chromium/WebGPU "
                               "adapter); CPU restatement of its WGSL kernels timed instead"},
            "cpu_baseline": {"value": value, "unit": "tok/s", "cores": cores, "kind": "port",
                             "sample": f"{per_step} greedy decode steps per step from position {prompt_len} "
                                       f"(the GPU arm's positions), C oracle fp32, {cores} OpenMP threads"},
            "e2e": {"value": value, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    m.close()


def decode_ids_check(cfg_name, path, ids, rank, sampling):
    """The first greedy ids after the prompt against the CPU oracle's, from
    the committed fixture (tests/golden/make_bench_fixture.py).  Only greedy
    configs on rank 0's prompt have a fixture; the model file's sha256 is
    compared first, so different model bytes are not reported as a parity
    failure."""
    fx_path = os.path.join(ROOT, "tests", "golden", "bench_decode_ids.json")
    try:
        with open(fx_path) as f:
            fx = json.load(f).get(cfg_name)
    except Exception:
        fx = None
    if fx is None or sampling or rank != 0:
        return {"match": None, "note": "no oracle fixture for this config"}
    import hashlib
    h = hashlib.sha256()
    with open(path, "rb") as f:
        for chunk in iter(lambda: f.read(1 << 24), b""):
            h.update(chunk)
    if h.hexdigest() != fx["gguf_sha256"]:
        return {"match": None, "note": "model bytes differ from the fixture's model"}
    n = min(len(fx["ids"]), len(ids))
    return {"match": list(ids[:n]) == fx["ids"][:n], "got": list(ids[:n]), "expected": fx["ids"][:n],
            "source": "CPU oracle, token-by-token prompt (tests/golden/bench_decode_ids.json)"}


def matvec_report(path, peak):
    """Matvec GB/s (algorithmic bytes: device-layout weights + 4k + 4n) of the
    streaming matvec kernel on the two large single-type matrices of the
    model, each launch streaming from HBM (copies rotated past L2): the tied
    LM head (Q6_K, 151936 x 1024 for Qwen3) and every layer's gate and up
    projections stacked into one Q4_K matrix."""
    from chonklm_b200 import _lib
    from chonklm_b200.gguf import ByteSource, fetch_gguf_header
    src = ByteSource(path)
    g = fetch_gguf_header(src)
    out = {}

    def one(label, t_type, k, n, data):
        us = _lib.bench_matvec(t_type, data, k, n, reps=50)
        dev_bytes = _lib.layout_row_bytes(t_type, k) * n
        byts = dev_bytes + 4 * k + 4 * n
        gbs = byts / (us * 1e-6) / 1e9
        out[label] = {"type": t_type, "k": k, "n": n, "MB": round(dev_bytes / 1e6, 1), "us": round(us, 2),
                      "GBps": round(gbs, 1), "frac": round(gbs / peak, 3)}

    t = g.tensor_map.get("output.weight") or g.tensor_map.get("token_embd.weight")
    if t is not None:
        one("lm_head", t.type, t.shape[0], t.shape[1], src.read(g.data_offset + t.offset, t.n_bytes))
    parts, rows, k, typ = [], 0, None, None
    for name, t in g.tensor_map.items():
        if name.endswith("ffn_gate.weight") or name.endswith("ffn_up.weight"):
            if typ is None:
                typ, k = t.type, t.shape[0]
            if t.type == typ and t.shape[0] == k:
                parts.append(src.read(g.data_offset + t.offset, t.n_bytes))
                rows += t.shape[1]
    if parts:
        one("gate_up_all_layers", typ, k, rows, b"".join(parts))
    return out


def phase_profile(eng, layers: int, start: int) -> dict:
    """CTA 0's view of one megakernel launch of a decode step (ck_trace
    globaltimer stamps around each phase, read after four traced steps): the
    mean duration of each phase kind over the layers.  A phase's time
    includes its wait for the previous phase's slowest producer.  The LM head,
    argmax stage 1 and select run as their own launches after the megakernel."""
    import numpy as np
    eng.truncate(start)              # the traced steps decode from the prompt end
    eng.trace(True)
    eng.enqueue_decode_steps(4)
    eng.sync()
    tr = eng.trace_read(4096).astype(np.int64)
    eng.trace(False)
    n = 0
    while n < 2048 and tr[2 * n] != 0:
        n += 1
    dur = (tr[1:2 * n:2] - tr[0:2 * n:2]) / 1000.0
    kinds = ["qkv", "attn", "o", "gate_up", "down"]
    if n != 1 + 5 * layers + 1:
        return {"phases": n, "total_us": round(float(dur.sum()), 1)}
    per = {k: round(float(np.mean(dur[1 + j:1 + 5 * layers:5])), 2) for j, k in enumerate(kinds)}
    return {"phases": n, "megakernel_us": round(float((tr[2 * n - 1] - tr[0]) / 1000.0), 1),
            "per_layer_mean_us": per, "embed_us": round(float(dur[0]), 2),
            "final_norm_us": round(float(dur[n - 1]), 2)}


def run_gemma_text(args, rank: int, world: int, barrier, local: int, dist) -> None:
    """Config 4's model through the text API (gemma-runtime.ts interface,
    chonklm_b200.gemma_runtime): a fixed user message, 256 sampled ids
    (temperature 1, top-k 64, top-p 0.95), tok/s as generateGemma reports it
    (generated ids over the time of the call, prompt prefill included)."""
    import torch
    from chonklm_b200.gemma_runtime import generateGemma, loadGemmaModel, resetGemmaConversation
    from chonklm_b200.registry import ModelDef
    torch.cuda.set_device(local)
    path = model_file("gemma3-270m", rank, world, barrier, tokenizer=True)
    loaded = loadGemmaModel(ModelDef(id="gemma3-270m-text", label="gemma3-270m-text", runtime="gemma-webgpu",
                                     maxContext=MAX_CONTEXT["gemma3-270m"], gguf=path), device=local)
    history = [{"role": "user", "content": "please answer the question about the world model " * 4}]
    opts = {"maxNewTokens": 256, "temperature": 1.0}
    vals = []
    for i in range(args.warmup + args.steps):
        resetGemmaConversation(loaded)
        r = generateGemma(loaded, history, opts)
        if i >= args.warmup:
            vals.append((r["tokensPerSec"], r["generatedTokens"]))
    barrier()
    tps = torch.tensor([statistics.median(v[0] for v in vals)], dtype=torch.float64, device="cuda")
    if dist is not None:
        dist.all_reduce(tps, op=dist.ReduceOp.SUM)
    if rank == 0:
        v = float(tps[0])
        print(json.dumps({"metric": "gemma text API tok/s (generateGemma, 256 sampled ids)", "value": round(v, 2),
                          "unit": "tok/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
                          "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
                          "dtype": "int8-dp4a/fp32", "data": "synthetic",
                          "config": {"workload": "gemma3-270m-text",
                                     "prompt_ids": len(loaded.engine.history_ids) - len(loaded.engine.last_reply_ids),
                                     "generated": 256, "sampling": "T 1.0, top-k 64, top-p 0.95, Philox seed 0",
                                     "parallelism": f"replicas x{world}"},
                          "e2e": {"value": round(v, 2), "unit": "tok/s", "h2d_bytes_per_step": None,
                                  "d2h_bytes_per_step": None},
                          "generated_last": vals[-1][1]}), flush=True)
    loaded.engine.dispose()


def shard(n: int, rank: int, world: int):
    """Sequences of the batched workload on this rank: i mod world == rank
    (independent sequences, no collective on the data path)."""
    return [i for i in range(n) if i % world == rank]


def aggregate(dist, seconds: float, generated: float, device: str = "cuda"):
    """Whole-job figures over ranks: the slowest rank's time, the sum of the
    tokens all ranks generated (every rank takes the same collective steps)."""
    import torch
    t = torch.tensor([seconds], dtype=torch.float64, device=device)
    g = torch.tensor([generated], dtype=torch.float64, device=device)
    if dist is not None:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        dist.all_reduce(g, op=dist.ReduceOp.SUM)
    return float(t[0]), float(g[0])


def run_batched(rank: int, world: int, barrier, local: int, warmup: int, max_steps: int = 0):
    """Config 5 on this rank's share of the sequences: every step advances
    each running sequence one position (ck_batch_step, host-synchronised);
    returns (generated tokens, seconds, steps, tokens fed)."""
    import numpy as np
    from chonklm_b200 import _lib
    from chonklm_b200.registry import ModelDef
    from chonklm_b200.runtime import loadLlamaWgslModel
    from chonklm_b200.synth import SPECS
    B = BATCHED
    S = SPECS[B["spec"]]
    path = model_file(B["spec"], rank, world, barrier)
    loaded = loadLlamaWgslModel(ModelDef(id="batched", label="batched", vocab=S.vocab, maxContext=B["max_context"],
                                         gguf=path, eosIds=[]), device=local)
    eng = loaded.engine.dev
    mine = shard(B["seqs"], rank, world)
    prompts = {i: np.random.default_rng(1 + i).integers(0, S.vocab, size=B["prompt"]).tolist() for i in mine}
    # warm-up: the same shapes on a throw-away batch (kernel loading, graph capture)
    wb = _lib.Batch(eng, max_seqs=len(mine))
    for i in mine:
        wb.add(prompts[i], B["generated"])
    for _ in range(warmup):
        wb.step()
    wb.close()
    b = _lib.Batch(eng, max_seqs=len(mine))
    for i in mine:
        b.add(prompts[i], B["generated"])
    barrier()
    t0 = time.perf_counter()
    n = 0
    while b.step() > 0:
        n += 1
        if max_steps and n >= max_steps:   # profiling runs stop early
            break
    dt = time.perf_counter() - t0
    steps, fed, gen = b.stats()
    b.close()
    loaded.engine.dispose()
    return gen, dt, steps, fed


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--config", default="qwen3-0.6b-q4_k_m",
                    choices=list(CONFIGS) + ["smollm2-135m-batched", "gemma3-270m-text"])
    ap.add_argument("--no-batched", action="store_true", help="skip the batched (config 5) summary")
    ap.add_argument("--mode", type=int, default=0, help="0 megakernel, 1 per-phase CUDA graph")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-matvec", action="store_true")
    ap.add_argument("--no-prefill", action="store_true", help="skip the prefill comparison")
    ap.add_argument("--prefill-profile", type=int, default=0, metavar="N",
                    help="profiling run for ncu: N tensor-core prefills of the config's prompt (the first one "
                         "formats the operand tiles), then exit")
    ap.add_argument("--matvec-profile", type=int, default=0, metavar="N",
                    help="profiling run for ncu: N launches of the streaming matvec kernel on the config's LM "
                         "head (copies rotated past L2), then exit")
    ap.add_argument("--profile", type=int, default=0, metavar="N",
                    help="profiling run for ncu: prefill the prompt (megakernel), decode N tokens in --mode, "
                         "print nothing else")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    import torch
    dist = None
    if world > 1:
        import datetime
        import torch.distributed as dist
        backend = "nccl" if torch.cuda.is_available() else "gloo"
        if backend == "nccl":
            torch.cuda.set_device(local)
        dist.init_process_group(backend, timeout=datetime.timedelta(seconds=600))

    def barrier():
        if dist is not None:
            dist.barrier()

    if args.impl == "reference":
        if args.config == "smollm2-135m-batched":
            if rank == 0:
                print(json.dumps({"impl": "reference", "unavailable":
                                  "the reference decodes one sequence per engine (no batched path) and its "
                                  "WebGPU runtime is unavailable on this box"}), flush=True)
        else:
            run_reference(args, args.config, rank, world, barrier)
        if dist is not None:
            dist.destroy_process_group()
        return

    if args.config == "gemma3-270m-text":
        if args.impl == "reference":
            if rank == 0:
                print(json.dumps({"impl": "reference", "unavailable":
                                  "the reference's gemma-webgpu engine is a third-party WebGPU package, absent "
                                  "here; no WebGPU on this box"}), flush=True)
        else:
            run_gemma_text(args, rank, world, barrier, local, dist)
        if dist is not None:
            dist.destroy_process_group()
        return

    if args.config == "smollm2-135m-batched":
        torch.cuda.set_device(local)
        gen, dt, steps, fed = run_batched(rank, world, barrier, local, args.warmup, args.profile)
        max_s, total_gen = aggregate(dist, dt, float(gen))
        if rank == 0:
            B = BATCHED
            print(json.dumps({
                "metric": BATCHED_METRIC, "value": round(total_gen / max_s, 1), "unit": "tok/s", "n_gpus": world,
                "steps": int(steps), "warmup": args.warmup, "ms_per_step": round(1000 * max_s / max(steps, 1), 4),
                "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "fp16x2/fp32-tcgen05",
                "data": "synthetic",
                "config": {"workload": "smollm2-135m-batched", "sequences": B["seqs"], "prompt": B["prompt"],
                           "generated": B["generated"], "kv_cache": "paged fp16, 16-position blocks",
                           "parallelism": f"sequences sharded over {world} GPU(s), no collective",
                           "timing": "wall clock over host-synchronised steps (each step: ids up, next ids down)"},
                "e2e": {"value": round(total_gen / max_s, 1), "unit": "tok/s",
                        "h2d_bytes_per_step": int(12 * B["seqs"] / world + 4),
                        "d2h_bytes_per_step": int(4 * B["seqs"] / world + 4)},
                "tokens_fed": int(fed), "tokens_generated": int(total_gen)}), flush=True)
        if dist is not None:
            dist.barrier()
            dist.destroy_process_group()
        return

    torch.cuda.set_device(local)
    spec, prompt_len, gen, sampling = CONFIGS[args.config]
    from chonklm_b200 import _lib
    from chonklm_b200.registry import ModelDef
    from chonklm_b200.runtime import generateLlamaWgsl, loadLlamaWgslModel, resetLlamaWgslConversation
    from chonklm_b200.synth import SPECS
    import numpy as np

    path = model_file(spec, rank, world, barrier)
    S = SPECS[spec]
    mdef = ModelDef(id=args.config, label=args.config, vocab=S.vocab, layers=S.layers, kvHeads=S.kv_heads,
                    headDim=S.head_dim, maxContext=MAX_CONTEXT[spec], gguf=path, eosIds=[])
    t = time.time()
    loaded = loadLlamaWgslModel(mdef, device=local)
    log(f"[bench r{rank}] loaded in {time.time() - t:.1f}s")
    eng = loaded.engine.dev
    eng.set_mode(args.mode)
    # a real (non-default) stream shared by the engine and the timing events
    stream = torch.cuda.Stream()
    eng.set_stream(stream.cuda_stream)
    prompt = np.random.default_rng(1 + rank).integers(0, S.vocab, size=prompt_len).tolist()
    samp = None
    if sampling:
        samp, _ = _lib.make_sampling(sampling["temperature"], sampling["topP"], sampling["topK"], 1.0,
                                     sampling["seed"], 0)
    if args.prefill_profile:
        eng.set_prefill_gemm(64)
        for _ in range(args.prefill_profile):
            eng.truncate(0)
            nid = eng.prefill(prompt, True, samp)
        print(json.dumps({"prefill_profile": args.config, "prefills": args.prefill_profile, "tokens": prompt_len,
                          "next_id": int(nid)}), flush=True)
        loaded.engine.dispose()
        return
    if args.matvec_profile:
        from chonklm_b200.gguf import ByteSource, fetch_gguf_header
        src = ByteSource(path)
        g = fetch_gguf_header(src)
        t = g.tensor_map.get("output.weight") or g.tensor_map.get("token_embd.weight")
        us = _lib.bench_matvec(t.type, src.read(g.data_offset + t.offset, t.n_bytes), t.shape[0], t.shape[1],
                               reps=args.matvec_profile)
        print(json.dumps({"matvec_profile": args.config, "type": t.type, "k": t.shape[0], "n": t.shape[1],
                          "launches": args.matvec_profile, "us": round(us, 2)}), flush=True)
        loaded.engine.dispose()
        return
    if args.profile:
        eng.set_mode(0)
        nid = eng.prefill(prompt, True, samp)
        eng.set_mode(args.mode)
        eng.enqueue_decode_steps(args.profile)
        eng.sync()
        print(json.dumps({"profile": args.config, "mode": args.mode, "tokens": args.profile,
                          "position": eng.position}), flush=True)
        loaded.engine.dispose()
        return
    nid = eng.prefill(prompt, True, samp)
    ids0 = eng.decode(nid, 8, samp)           # stores the first id at the prompt end
    eng.truncate(prompt_len)
    w0, kv0 = eng.step_bytes()
    eng.truncate(prompt_len)

    # L2 (126 MB) is flushed before every step, outside the timed events, by
    # writing a 256 MB buffer on the step's stream: a model whose weights fit
    # in L2 (SmolLM2, ~107 MB) starts each step from HBM like the others
    l2_flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")

    def one_step():
        eng.truncate(prompt_len)
        with torch.cuda.stream(stream):
            l2_flush.fill_(1)
        ev0 = torch.cuda.Event(enable_timing=True)
        ev1 = torch.cuda.Event(enable_timing=True)
        ev0.record(stream)
        eng.enqueue_decode_steps(gen, samp)      # the config's sampling, as the e2e arm runs it
        ev1.record(stream)
        return ev0, ev1

    for _ in range(args.warmup):
        one_step()
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    evs = []
    with Clocks(local) as clk:
        for _ in range(args.steps):
            evs.append(one_step())
        torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    eng.sync()
    step_ms = [a.elapsed_time(b) for a, b in evs]
    tot_ms = sum(step_ms)
    # KV bytes per token averaged over the step's positions
    eng.truncate(prompt_len + gen - 1)
    w1, kv1 = eng.step_bytes()
    bytes_per_token = w0 + 0.5 * (kv0 + kv1)

    phases = phase_profile(eng, S.layers, prompt_len) if (rank == 0 and args.mode == 0) else None

    # ---- e2e through generateLlamaWgsl -------------------------------------
    e2e_times = []
    e2e_io = []
    opts = {"maxNewTokens": gen}
    if sampling:
        opts.update(sampling)
    for i in range(args.warmup + args.steps):
        loaded.cachedTokenIds = list(prompt)
        loaded.cachedNextId = nid
        eng.truncate(prompt_len)
        io0 = eng.io_bytes()
        t0 = time.perf_counter()
        res = generateLlamaWgsl(loaded, prompt, opts)
        dt = time.perf_counter() - t0
        io1 = eng.io_bytes()
        if i >= args.warmup:
            e2e_times.append(dt)
            e2e_io.append((io1[0] - io0[0], io1[1] - io0[1]))
        assert len(res["ids"]) == gen, len(res["ids"])

    # ---- prefill: tensor-core path against token by token -------------------------
    prefill = None
    if rank == 0 and not args.no_prefill:
        def time_prefill(min_tokens):
            eng.set_prefill_gemm(min_tokens)
            eng.truncate(0)
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            eng.prefill(prompt, True, samp)        # returns after the device finished
            return 1000.0 * (time.perf_counter() - t0)
        pf_ms = [time_prefill(64) for _ in range(4)][1:]   # the first call formats the operand tiles
        tbt_ms = time_prefill(0)
        eng.set_prefill_gemm(64)
        # the reference's tok/s: generated ids over the time from before the
        # prefill (llama-wgsl-runtime.ts:266, :312), fresh conversation each run
        ref_def = []
        for _ in range(2):
            resetLlamaWgslConversation(loaded)
            t0 = time.perf_counter()
            res = generateLlamaWgsl(loaded, prompt, opts)
            ref_def.append(len(res["ids"]) / (time.perf_counter() - t0))
        prefill = {"tokens": prompt_len, "tensor_core_ms": round(statistics.median(pf_ms), 2),
                   "tensor_core_tok_per_s": round(prompt_len / (statistics.median(pf_ms) / 1000.0), 1),
                   "token_by_token_ms": round(tbt_ms, 2),
                   "generate_tok_per_s_from_before_prefill": round(max(ref_def), 2),
                   "note": "ck_prefill host-synchronised wall time; all but the last prompt id through "
                           "tcgen05 GEMMs + flash attention (prompts >= 64 ids)"}
        eng.truncate(prompt_len)

    # ---- reduce over ranks ------------------------------------------------------
    vals = torch.tensor([tot_ms, sum(e2e_times)], dtype=torch.float64, device="cuda")
    if dist is not None:
        dist.all_reduce(vals, op=dist.ReduceOp.MAX)
    max_ms, max_e2e = float(vals[0]), float(vals[1])

    # ---- batched workload at this N: sequence i on rank
    # i mod N, no collective on the data path; every rank takes part ----------
    batched = None
    if not args.no_batched:
        gen_b, dt_b, steps_b, fed_b = run_batched(rank, world, barrier, local, 3)
        max_b, total_b = aggregate(dist, dt_b, float(gen_b))
        steps_t = torch.tensor([float(steps_b)], dtype=torch.float64, device="cuda")
        if dist is not None:
            dist.all_reduce(steps_t, op=dist.ReduceOp.MAX)
        B = BATCHED
        batched = {"metric": BATCHED_METRIC, "value": round(total_b / max_b, 1), "unit": "tok/s", "n_gpus": world,
                   "scaling": "strong", "sequences": B["seqs"], "sequences_per_gpu": -(-B["seqs"] // world),
                   "ms_per_step": round(1000 * max_b / max(float(steps_t[0]), 1), 3),
                   "steps": int(steps_t[0]), "tokens_generated": int(total_b),
                   "config": "smollm2-135m-batched (BASELINE configs[4]): 256 x (128 prompt + 256 greedy), "
                             f"sequences sharded over {world} GPU(s) (i mod N), slowest rank's wall time"}
    tokens = gen * args.steps * world
    value = tokens / (max_ms / 1000.0)
    e2e_value = tokens / max_e2e

    out = None
    check = decode_ids_check(args.config, path, ids0, rank, sampling) if rank == 0 else None
    if rank == 0:
        peak, peak_kind = peaks()
        per_tok_s = (tot_ms / 1000.0) / (gen * args.steps)
        achieved = bytes_per_token / per_tok_s / 1e9
        # DRAM bytes (read + write) of one launch of the dominant kernel, from the
        # committed ncu capture of this workload (profiles/); null when absent
        traffic, traffic_note = None, None
        try:
            with open(os.path.join(ROOT, "profiles", "traffic.json")) as f:
                t = json.load(f).get(args.config)
            if t and args.mode == 0:
                traffic = t["bytes_per_launch"]
                traffic_note = (f"ncu dram__bytes_read+write of one decode step ({t['kernel']}, the step's "
                                f"weight- and KV-streaming launches) at position {t['position']}")
        except Exception:
            traffic = None
        cpu = None
        if world == 1 and not args.no_cpu_baseline:
            try:
                cpu = cpu_baseline_sample(path, S.vocab, MAX_CONTEXT[spec], prompt_len)
            except Exception as e:  # reported, not fatal
                cpu = {"value": None, "error": str(e)}
        mv = None
        if not args.no_matvec:
            try:
                mv = matvec_report(path, peak)
            except Exception as e:
                mv = {"error": str(e)}
        # megakernel mode: the megakernel, the LM head, argmax stage 1, select;
        # graph mode: embed, 5 per layer, final norm, head, argmax stage 1, select
        launches_per_token = 4 if args.mode == 0 else 1 + 5 * S.layers + 4
        out = {
            "metric": METRIC, "value": round(value, 2), "unit": "tok/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(tot_ms / args.steps, 4), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "int8-dp4a/fp32", "data": "synthetic",
            "config": {"workload": args.config, "prompt": prompt_len, "generated": gen,
                       "weights": "N(0,0.02) seed 0, Q4_K_M mixture", "kv_cache": "fp16",
                       "mode": "megakernel" if args.mode == 0 else "graph",
                       "l2": ("L2 flushed before every timed step (256 MB write); weights %.0f MB per token %s "
                              "126 MB L2, re-read by each of the step's %d tokens"
                              % (w0 / 1e6, ">" if w0 > 126e6 else "<", gen)),
                       "parallelism": f"replicas x{world}",
                       "sampling": (dict(sampling, sampler="chunk maxima (sampleFromCandidateBuffer)")
                                    if sampling else "greedy")},
            "e2e": {"value": round(e2e_value, 2), "unit": "tok/s",
                    "h2d_bytes_per_step": int(statistics.mean(x[0] for x in e2e_io)),
                    "d2h_bytes_per_step": int(statistics.mean(x[1] for x in e2e_io)),
                    "note": "generateLlamaWgsl wall time; its 256 ids take 255 device steps (the first id "
                            "is the one the prompt's last step produced, reused as the reference does), so "
                            "e2e can come within a step of value or pass it"},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "traffic": traffic, "traffic_note": traffic_note,
                         "peak_source": peak_kind,
                         "bytes_per_token": round(bytes_per_token), "us_per_token": round(per_tok_s * 1e6, 2)},
            "cpu_baseline": cpu,
            "matvec": mv,
            "batched": batched,
            "prefill": prefill,
            "phases": phases,
            "clocks": clk.summary(),
            "gpu_launches": int(launches_per_token * gen * args.steps),
            "decode_ids_head": ids0[:8],
            "decode_ids_check": check,
        }
        print(json.dumps(out), flush=True)
    loaded.engine.dispose()
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()
    if check is not None and check.get("match") is False:
        log("[bench] PARITY FAILURE: the decoded ids differ from the CPU oracle's "
            f"(tests/golden/bench_decode_ids.json): got {check['got']}, expected {check['expected']}")
        sys.exit(3)


if __name__ == "__main__":
    main()
