"""Benchmark: batch-1 decode of the Llama-2-7B-shape Q4_0 model on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload llama7b_q4_0|llama7b_q8_0|llama70b_q4_0|stories_f32] [--layers L]

--layers L keeps the workload's shapes with L layers (a small case for
profiling; the workload name then carries the layer count).

One step = one decode token: every layer's rmsnorm + quantize + qkv matvec +
RoPE, attention over the KV cache, wo, w1/w3 + SwiGLU, w2, then the classifier
and the greedy argmax (cats_llama2_transformer, llm/catseye_llm.h:1625-1772).
Synthetic weights N(0, 0.02) quantized per 32-block (generated on the device);
the 3.7 GB of weights exceed the 126 MB L2, so every step streams them from
HBM (no L2 flush needed).

value : tokens/s of K greedy steps run by one launch of the persistent decode
        kernel (argmax fed back on the device, inputs resident in HBM), timed
        with CUDA events on the model's stream.
e2e   : tokens/s through the public C API cats_gpu_llama2_transformer(token,
        pos, m, logits) — token/pos copied in, the logits copied out, every step.
roofline : that kernel (it is the whole step): algorithmic bytes (every weight
        once per step + the K/V rows attention reads) / its event-timed duration.
cpu_baseline : the reference's own CPU step (oracle/_ref, OpenMP on every
        host core) on the full model at its own context, 12 real greedy
        steps after the prompt (a model larger than the host's free memory:
        a quarter and a half of its layers, per-layer slope stated).

vs_baseline : value / the reference's own published decode rate of the same
        model shape and weight type (llm/README.md:259: Llama-2-7B-chat GGUF
        Q4_0, 5.47 tok/s on a CPU whose hardware it does not state), named in
        vs_baseline_of; null for the workloads it publishes nothing for.

--impl reference times only that CPU reference on the same workload.

--workload llama70b_q4_0_prefill512 | llama7b_q4_0_batch16 measure the
batched step on the tensor cores (cats_gpu_llm_forward_batch): a 512-token
prompt prefilled through the 80-layer Llama-2-70B-shape Q4_0 model in one
step (value = prompt tok/s), or 16 sequences decoded one token each per step
on the 7B shape (value = tok/s over all 16; the step is a CUDA graph replayed
with the argmax fed back on the device).  roofline: the tcgen05 product
(k_qgemm) of the largest weight (w1/w3) at the step's token count, timed on
its own with CUDA events: tensor FLOP/s against the measured bf16 peak for
prefill, weight bytes/s against the measured HBM copy rate for batch 16.
e2e = the host API (token ids in, argmax ids out); cpu_baseline = the
reference's own step on all cores (it processes a prompt or a batch one
token at a time, so its tok/s is its decode rate).

--workload sgemm_4096 | cnn_forward_b128 measure the CNN side instead: a
4096^3 fp32 NN sgemm (cats_sgemm_dev), or the 32x32x3 CNN's four
convolutions and two linear layers at batch 128 (cats_conv2d_forward_dev /
cats_linear_forward_dev, 25.15 GFLOP).  value = GFLOP/s on device buffers;
e2e = the host-pointer API with its copies; roofline against the 3xTF32
tensor peak (the measured bf16 peak / 2 for tf32 / 3 products per fp32
product), since both run on k_sgemm_tc; cpu_baseline = the reference's gemm_rnn / layer forwards
(oracle/_ref, OpenMP on all cores) on a bounded sample.
With torchrun (N > 1) the N ranks hold one model sharded by tensor
parallelism (wq/wk/wv and w1/w3 by rows, wo and w2 by input columns, the
classifier by vocabulary rows) and decode one sequence in the persistent
kernel, the partial rows of wo and w2 pushed to every rank over NVLink
(value = that sequence's tokens/s, "strong" scaling; roofline per GPU over
the rank's weight slice).  Before timing, rank 0 runs the same model
unsharded and the line's `parity` compares the prompt steps' logits.
torch.distributed runs on gloo and only shares the NCCL id, aligns the
ranks and takes the max of their times.  --replicas runs N independent
copies instead (value = the tokens of all ranks, "weak").
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

WORKLOADS = {
    "llama7b_q4_0": ("LLAMA2_7B", 2),
    "llama7b_q8_0": ("LLAMA2_7B", 8),
    "llama70b_q4_0": ("LLAMA2_70B", 2),
    "stories_f32": ("STORIES_F32", 0),
}
PROMPT = 8
SEED = 20241201
# The reference's own published decode rate for the same model shape and
# weight type (CPU, hardware not stated): the denominator of vs_baseline.
PUBLISHED = {"llama7b_q4_0": (5.47, "llm/README.md:259, Llama-2-7B-chat GGUF Q4_0 decode on a CPU")}


def vs_published(args, value):
    """value / the published rate of this exact workload (full layer count), else None."""
    pub = PUBLISHED.get(args.workload)
    return round(value / pub[0], 2) if pub and not args.layers else None


def cfg_for(workload, layers=0):
    from dataclasses import replace
    from catseye_b200 import llm
    name, t = WORKLOADS[workload]
    cfg = getattr(llm, name).with_type(t)
    return replace(cfg, n_layers=layers) if layers else cfg


def workload_name(args):
    return args.workload + (f"_{args.layers}layers" if args.layers else "")


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def tensor_peak():
    """Dense bf16 tensor peak (TFLOP/s): the measured cuBLAS burst figure."""
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        return float(json.load(open(p))["bf16_tflops"]), "measured (cuBLAS bf16 burst)"
    return 1590.0, "fallback"


# batched workloads: (model, weight type, tokens per step, sequences)
BATCHED = {
    "llama70b_q4_0_prefill512": ("LLAMA2_70B", 2, 512, 1),
    "llama7b_q4_0_batch16": ("LLAMA2_7B", 2, 16, 16),
}


class Clocks:
    """nvidia-smi sampling during the timed region (clocks + throttle reasons)."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, device):
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        self.device = device
        self.p = None

    def __enter__(self):
        try:
            self.p = subprocess.Popen(["nvidia-smi", "-i", str(self.device), f"--query-gpu={self.Q}",
                                       "--format=csv,noheader,nounits", "-lms", "25"],
                                      stdout=self.f, stderr=subprocess.DEVNULL)
        except OSError:
            self.p = None
        time.sleep(0.3)
        return self

    def __exit__(self, *a):
        if self.p:
            self.p.terminate()
            try:
                self.p.wait(5)
            except subprocess.TimeoutExpired:
                self.p.kill()

    def summary(self):
        self.f.flush()
        rows = []
        try:
            for line in open(self.f.name):
                parts = [s.strip() for s in line.split(",")]
                if len(parts) >= 9 and parts[1].replace(".", "").isdigit():
                    rows.append(parts)
        finally:
            os.unlink(self.f.name)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[1]) for r in rows]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower().startswith("active")})
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": float(rows[0][2]), "reasons": reasons,
                "samples": len(rows)}


def dist_init(backend="nccl"):
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if ws == 1:
        return None, 0, 1, int(os.environ.get("LOCAL_RANK", "0"))
    import datetime
    import torch
    import torch.distributed as dist
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if backend == "nccl":
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    else:
        dist.init_process_group(backend, timeout=datetime.timedelta(seconds=120))
    return dist, rank, ws, local


# ------------------------------------------------------------- CPU reference
def _omp_all_cores():
    """The reference's OpenMP loops on every host core: torchrun exports
    OMP_NUM_THREADS=1, which would otherwise leave the reference one thread."""
    import ctypes
    n = os.cpu_count() or 1
    os.environ["OMP_NUM_THREADS"] = str(n)
    try:
        ctypes.CDLL("libgomp.so.1").omp_set_num_threads(n)
    except (OSError, AttributeError):
        pass
    return n


def _host_timing_model(cfg, orc, layers):
    """A host model with the workload's shapes for timing the reference step:
    one seeded layer of N(0, 0.02) weights quantized like the GPU model's,
    copied into `layers` separate layers (every layer's weights are distinct
    memory, so each step streams all of them; the dot products' cost does not
    depend on the values)."""
    from dataclasses import replace
    from oracle.models import ModelWeights
    one = ModelWeights(replace(cfg, n_layers=1), SEED, orc)

    class MW:
        pass
    mw = MW()
    mw.cfg = replace(cfg, n_layers=layers)
    mw.emb, mw.rms_final, mw.wcls = one.emb, one.rms_final, one.wcls
    mw.rms_att = np.ones((layers, cfg.dim), np.float32)
    mw.rms_ffn = np.ones((layers, cfg.dim), np.float32)
    from oracle.cpu import aligned
    for k in ("wq", "wk", "wv", "wo", "w1", "w2", "w3"):
        blob = getattr(one, k)
        out = aligned(np.empty(blob.size * layers, blob.dtype))   # the reference's 256-byte alignment, no copy later
        out.reshape(layers, blob.size)[:] = blob
        setattr(mw, k, out)
    return mw


def _host_mem_available():
    try:
        for line in open("/proc/meminfo"):
            if line.startswith("MemAvailable:"):
                return int(line.split()[1]) * 1024
    except OSError:
        pass
    return 0


def cpu_reference(cfg, kind="reference", tokens=12):
    """Time the reference's own decode step (cats_llama2_transformer, oracle/_ref
    built for all cores) on the host cores, for `tokens` real steps of the
    workload's model at its own context length, after 8 prompt steps.

    A model too large for the host's free memory is timed at two layer counts
    far apart (a quarter and a half of its layers): per token = t_a + (L - L_a)
    * (t_b - t_a) / (L_b - L_a), stated in `sample`."""
    from dataclasses import replace
    from catseye_b200 import llm
    from oracle.cpu import Oracle, Reference, ref_available
    cores = _omp_all_cores()
    orc = Oracle()
    use_ref = kind == "reference" and ref_available("llm_allcores") and cfg.wtype in (0, 2)
    full = llm.weight_bytes(cfg) + 2 * cfg.n_layers * cfg.seq_len * cfg.kv_dim * 4
    fits = full * 1.3 < _host_mem_available() or full < 8e9

    def time_model(L):
        mw = _host_timing_model(cfg, orc, L)
        m = Reference("llm_allcores").llm(mw) if use_ref else orc.llm(mw)
        rng = np.random.default_rng(SEED + 1)
        tok = 0
        for pos, t in enumerate(rng.integers(0, cfg.vocab, PROMPT)):   # prompt, untimed
            tok = int(np.argmax(m.step(int(t), pos)))
        t0 = time.perf_counter()
        for i in range(tokens):
            tok = int(np.argmax(m.step(tok, PROMPT + i)))
        dt = (time.perf_counter() - t0) / tokens
        del m, mw
        return dt

    if fits:
        t_tok = time_model(cfg.n_layers)
        sample = (f"full {cfg.n_layers}-layer model (context {cfg.seq_len}), {tokens} greedy steps at positions "
                  f"{PROMPT}-{PROMPT + tokens - 1} after an {PROMPT}-token prompt: {t_tok * 1e3:.1f} ms per token")
    else:
        la, lb = max(1, cfg.n_layers // 4), max(2, cfg.n_layers // 2)
        ta, tb = time_model(la), time_model(lb)
        t_tok = ta + (cfg.n_layers - la) * (tb - ta) / (lb - la)
        sample = (f"{la}- and {lb}-layer models (context {cfg.seq_len}; the full model exceeds the host's free "
                  f"memory), {tokens} greedy steps each; per token = t{la} + {cfg.n_layers - la} x (t{lb} - t{la}) "
                  f"/ {lb - la} = {t_tok * 1e3:.1f} ms")
    return {"value": 1.0 / t_tok, "unit": "tok/s", "cores": cores,
            "kind": "reference" if use_ref else "port", "sample": sample}


def decode_config(args, cfg, ws, tp):
    """The `config` object of a decode line, the same in both arms."""
    from catseye_b200 import llm
    wbytes = llm.weight_bytes(cfg)
    return {"workload": workload_name(args), "batch": 1, "prompt": PROMPT, "dim": cfg.dim,
            "layers": cfg.n_layers, "context": cfg.seq_len,
            "parallelism": f"tp{ws}" if tp else (f"replicas{ws}" if ws > 1 else "single"),
            "l2": (f"weights {wbytes / 1e9:.2f} GB per step > 126 MB L2; no flush" if wbytes > 126e6 else
                   f"weights {wbytes / 1e6:.0f} MB per step; L2-resident, no flush")}


# ------------------------------------------------------------------ our arm
PARITY_STEPS = 8


def tp_parity(args, cfg, dist, rank, prompt_logits):
    """Sharded model vs one GPU: rank 0 builds the unsharded model of the same
    seed on its own GPU, feeds it the same prompt and compares every step's
    logits (normwise) and greedy token with what the sharded ranks computed.
    The other ranks wait at the barrier."""
    from catseye_b200 import llm
    out = None
    if rank == 0:
        m = llm.GpuLLM(cfg)
        m.init_random(SEED)
        rng = np.random.default_rng(SEED + 1)
        errs, same = [], 0
        for pos, tok in enumerate(rng.integers(0, cfg.vocab, PROMPT)[:PARITY_STEPS]):
            lg = m.step(int(tok), pos)
            t = prompt_logits[pos]
            errs.append(float(np.linalg.norm(t - lg) / np.linalg.norm(lg)))
            same += int(np.argmax(t)) == int(np.argmax(lg))
        m.close()
        # quantized activations: a Q8 code rounding the other way after a float-order
        # difference moves the logits by up to a few 1e-2 (the reference's own AVX
        # and plain-C builds differ by 3-4e-2 on the 7B model).  Every layer
        # requantizes its inputs, so the flips add up layer by layer: measured
        # 1.34-1.44e-3 per layer (32-layer 7B over 2, 4, 8 ranks; 80-layer 70B over
        # 8), bar 1.9e-3 per layer.  fp32 models: 1e-4
        bar = 1e-4 if cfg.wtype == 0 else round(1.875e-3 * cfg.n_layers, 6)
        out = {"vs": "the same model unsharded on one GPU (seed %d), prompt steps 0-%d" % (SEED, PARITY_STEPS - 1),
               "max_rel": round(max(errs), 6), "bar": bar, "greedy_equal": f"{same}/{len(errs)}",
               "ok": bool(max(errs) < bar and (cfg.wtype != 0 or same == len(errs)))}
    if dist:
        dist.barrier()
    return out


def run_ours(args, dist, rank, ws, local):
    import torch
    from catseye_b200 import _lib, llm
    _lib.init(local)
    torch.cuda.set_device(local)
    cfg = cfg_for(args.workload, args.layers)
    tp = ws > 1 and not args.replicas
    if tp:
        m = llm.GpuLLM(cfg, rank, ws)
        m.tp_connect(llm.tp_share_id())
    else:
        m = llm.GpuLLM(cfg)
    engine = "persistent"
    if tp and not m.tp_persistent():
        m.set_engine(llm.ENGINE_GRAPH)
        engine = "graph"
    m.init_random(SEED)
    if dist:   # sharded: the ranks start their first step together (the exchange waits are bounded)
        dist.barrier()
    red_dev = "cpu" if tp else "cuda"     # gloo reduces host tensors
    stream = torch.cuda.ExternalStream(m.stream)
    rng = np.random.default_rng(SEED + 1)
    prompt = rng.integers(0, cfg.vocab, PROMPT)
    prompt_logits = []
    for pos, tok in enumerate(prompt):            # prompt forcing (untimed)
        prompt_logits.append(m.step(int(tok), pos).copy())
    parity = tp_parity(args, cfg, dist, rank, prompt_logits) if tp else None
    pos0 = PROMPT
    assert pos0 + args.warmup + args.steps + args.e2e_steps <= cfg.seq_len
    m.set_position(int(np.argmax(prompt_logits[-1])), pos0)
    m.enqueue(args.warmup)
    m.synchronize()

    def barrier():
        if dist:
            dist.barrier()

    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize()
    with Clocks(local) as clk:
        e0.record(stream)
        m.enqueue(args.steps)
        e1.record(stream)
        e1.synchronize()
    torch.cuda.synchronize()
    barrier()
    ms = e0.elapsed_time(e1)
    if dist:
        t = torch.tensor([ms], device=red_dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    clocks = clk.summary()
    pos = pos0 + args.warmup + args.steps

    # e2e through the public API: host token in, host logits out, every step
    tok = m.next_token()
    barrier()
    t0 = time.perf_counter()
    for i in range(args.e2e_steps):
        lg = m.step(tok, pos + i)
        tok = int(np.argmax(lg))
    e2e_s = time.perf_counter() - t0
    if dist:
        t = torch.tensor([e2e_s], device=red_dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_s = float(t.item())

    # per-phase kernels of the graph engine, timed alone (diagnostic)
    kinds = {}
    for k, name in enumerate(() if tp else ("qkv", "wo", "w13", "w2", "cls")):
        a, b = m.time_matvec(k, reps=2)
        kinds[name] = {"us_per_launch": round(a * 1e3, 2), "gbs": round(b / (a * 1e-3) / 1e9, 1)}
    wbytes = m.weight_bytes()
    m.close()
    # algorithmic bytes of the timed launch: every weight once per step, plus the
    # K and V rows 0..pos of every layer that attention reads
    kv_row = cfg.kv_dim * 4 // (ws if tp else 1)   # this rank's K/V heads
    kv_bytes = sum(2 * cfg.n_layers * kv_row * (p + 1) for p in range(pos0 + args.warmup, pos0 + args.warmup + args.steps))
    kbytes = wbytes * args.steps + kv_bytes
    return dict(ms=ms, e2e_s=e2e_s, kbytes=kbytes, kinds=kinds, wbytes=wbytes, clocks=clocks, cfg=cfg, tp=tp,
                engine=engine, parity=parity)


# -------------------------------------------- batched step (prefill, batch 16)
def run_batched(args, dist, rank, ws, local):
    import torch
    from catseye_b200 import _lib, llm
    _lib.init(local)
    torch.cuda.set_device(local)
    name, t, T, nseq = BATCHED[args.workload]
    cfg = getattr(llm, name).with_type(t)
    if args.layers:
        from dataclasses import replace
        cfg = replace(cfg, n_layers=args.layers)
    m = llm.GpuLLM(cfg)
    m.init_random(SEED)
    stream = torch.cuda.ExternalStream(m.stream)
    rng = np.random.default_rng(SEED + 1 + rank)
    prefill = nseq == 1
    if prefill:
        m.batch_reserve(T, 1)
        toks = rng.integers(0, cfg.vocab, T).astype(np.int32)
        pos = np.arange(T, dtype=np.int32)
        m.batch_set(toks, pos)
        launch = m.batch_enqueue
        step_tokens = T

        def host_step():
            return m.forward_batch(toks, pos)
        h2d, d2h = 3 * 4 * T, 4 * T
    else:
        m.batch_reserve(max(T, nseq * PROMPT), nseq)
        ptoks = rng.integers(0, cfg.vocab, nseq * PROMPT).astype(np.int32)
        ppos = np.tile(np.arange(PROMPT, dtype=np.int32), nseq)
        pseq = np.repeat(np.arange(nseq, dtype=np.int32), PROMPT)
        nxt = m.forward_batch(ptoks, ppos, pseq)           # every sequence's prompt, one call (untimed)
        first = nxt[PROMPT - 1::PROMPT].copy()
        p0 = np.full(nseq, PROMPT, np.int32)
        assert PROMPT + args.warmup + args.steps + args.e2e_steps <= cfg.seq_len
        m.batch_set(first, p0, np.arange(nseq, dtype=np.int32))
        step_tokens = nseq

        def launch(k=1):
            m.batch_enqueue_decode(k)
        state = {"tok": first, "pos": p0 + args.warmup + args.steps}

        def host_step():
            state["tok"] = m.forward_batch(state["tok"], state["pos"], np.arange(nseq, dtype=np.int32))
            state["pos"] = state["pos"] + 1
            return state["tok"]
        h2d, d2h = 3 * 4 * nseq, 4 * nseq

    def barrier():
        if dist:
            dist.barrier()

    if prefill:
        for _ in range(args.warmup):
            launch()
    else:
        launch(args.warmup)
    torch.cuda.synchronize()
    m.synchronize()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(local) as clk:
        e0.record(stream)
        if prefill:
            for _ in range(args.steps):
                launch()
        else:
            launch(args.steps)
        e1.record(stream)
        e1.synchronize()
    torch.cuda.synchronize()
    m.synchronize()
    barrier()
    ms = e0.elapsed_time(e1)
    if dist:
        tt = torch.tensor([ms], device="cuda")
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        ms = float(tt.item())
    clocks = clk.summary()
    e2e_steps = max(1, min(args.e2e_steps, 4 if prefill else args.e2e_steps))
    host_step()
    barrier()
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        host_step()
    e2e_s = time.perf_counter() - t0
    if dist:
        tt = torch.tensor([e2e_s], device="cuda")
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        e2e_s = float(tt.item())
    # the products timed alone at this token count (diagnostic + roofline)
    kinds = {}
    for k, kname in enumerate(("qkv", "wo", "w13", "w2", "cls")):
        kms, fl, wb = m.time_product(k, T, reps=2)
        kinds[kname] = {"us_per_launch": round(kms * 1e3, 2), "tflops": round(fl / (kms * 1e-3) / 1e12, 1),
                        "weight_gbs": round(wb / (kms * 1e-3) / 1e9, 1), "flop": fl, "weight_bytes": wb}
    wbytes = m.weight_bytes()
    m.close()
    return dict(ms=ms, e2e_s=e2e_s, e2e_steps=e2e_steps, kinds=kinds, wbytes=wbytes, clocks=clocks, cfg=cfg, T=T,
                nseq=nseq, step_tokens=step_tokens, h2d=h2d, d2h=d2h, prefill=prefill)


def batched_main(args):
    name, t, T, nseq = BATCHED[args.workload]
    prefill = nseq == 1
    metric = f"prefill tok/s ({T}-token prompt)" if prefill else f"decode tok/s (batch {nseq})"
    dtype = "q4_0 weights dequantized to f16 x f16 activations, f32 accumulate (tcgen05)"
    if args.impl == "reference":
        if int(os.environ.get("RANK", "0")) != 0:
            return
        from catseye_b200 import llm
        cfg = getattr(llm, name).with_type(t)
        cb = cpu_reference(cfg, "reference")
        cb["sample"] += "; the reference runs a prompt or a batch one token at a time, so this is its rate"
        print(json.dumps({"impl": "reference", "metric": metric, "value": round(cb["value"], 3), "unit": "tok/s",
                          "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "higher_is_better": True,
                          "scaling": "weak", "vs_baseline": None, "dtype": "q4_0 x q8 (int8 dot, f32 accumulate)",
                          "data": "synthetic", "config": {"workload": workload_name(args)}, "cpu_baseline": cb,
                          "e2e": {"value": round(cb["value"], 3), "unit": "tok/s", "h2d_bytes_per_step": 0,
                                  "d2h_bytes_per_step": 0}}))
        return
    dist, rank, ws, local = dist_init()
    r = run_batched(args, dist, rank, ws, local)
    if rank == 0:
        cfg, ms = r["cfg"], r["ms"]
        tok_s = ws * r["step_tokens"] * args.steps / (ms * 1e-3)
        w13 = r["kinds"]["w13"]
        kms = w13["flop"] / (w13["tflops"] * 1e12) * 1e3
        if prefill:
            peak, peak_kind = tensor_peak()
            achieved = w13["tflops"]
            roof = {"bound": "tensor", "kernel": f"k_qgemm (w1/w3 product, {cfg.dim}x{2 * cfg.hidden}, T={T})",
                    "achieved": achieved, "peak": peak, "peak_kind": peak_kind, "unit": "TFLOP/s",
                    "frac": round(achieved / peak, 4), "traffic": None, "flop_per_launch": w13["flop"],
                    "ms_per_launch": round(kms, 4)}
        else:
            peak, peak_kind = peaks()
            achieved = w13["weight_gbs"]
            roof = {"bound": "hbm", "kernel": f"k_qgemm (w1/w3 product, {cfg.dim}x{2 * cfg.hidden}, T={T})",
                    "achieved": achieved, "peak": peak, "peak_kind": peak_kind, "unit": "GB/s",
                    "frac": round(achieved / peak, 4), "traffic": None, "bytes_per_launch": w13["weight_bytes"],
                    "ms_per_launch": round(kms, 4)}
        step_flop = 2.0 * (r["wbytes"] / 18 * 32) * r["step_tokens"]
        launches = cfg.n_layers * 10 + (4 if prefill else 5)
        line = {"metric": metric, "value": round(tok_s, 2), "unit": "tok/s", "n_gpus": ws, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 4), "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None, "dtype": dtype, "data": "synthetic",
                "config": {"workload": workload_name(args), "tokens_per_step": r["step_tokens"], "sequences": nseq,
                           "dim": cfg.dim, "layers": cfg.n_layers, "heads": cfg.n_heads, "kv_heads": cfg.n_kv_heads,
                           "context": cfg.seq_len, "parallelism": f"replicas{ws}" if ws > 1 else "single",
                           "weight_tflop_per_s": round(step_flop * args.steps / (ms * 1e-3) / 1e12, 1),
                           "l2": f"weights {r['wbytes'] / 1e9:.1f} GB per step > 126 MB L2; no flush"},
                "roofline": roof, "products": {k: {kk: v[kk] for kk in ("us_per_launch", "tflops", "weight_gbs")}
                                               for k, v in r["kinds"].items()},
                "e2e": {"value": round(ws * r["step_tokens"] * r["e2e_steps"] / r["e2e_s"], 2), "unit": "tok/s",
                        "h2d_bytes_per_step": r["h2d"], "d2h_bytes_per_step": r["d2h"]},
                "gpu_launches": launches * args.steps, "clocks": r["clocks"]}
        if not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_reference(cfg, "reference")
        print(json.dumps(line))
    if dist:
        dist.destroy_process_group()


# ------------------------------------------------ fp32 GEMM workloads (CNN side)
# (kind, batch, ich|in, h, w, ch|out, ksize, pad, stride): the 32x32x3 CNN's
# four convolutions and two linear layers at batch 128 (25.15 GFLOP)
CNN_LAYERS = [("conv", 128, 3, 32, 32, 64, 3, 1, 1), ("conv", 128, 64, 32, 32, 64, 3, 1, 1),
              ("conv", 128, 64, 16, 16, 128, 3, 1, 1), ("conv", 128, 128, 16, 16, 128, 3, 1, 1),
              ("linear", 128, 8192, 0, 0, 256, 0, 0, 0), ("linear", 128, 256, 0, 0, 10, 0, 0, 0)]
SGEMM_SIZE = 4096


def _conv_out(n, k, pad, stride):
    return (n + 2 * pad - k) // stride + 1


def layer_flops(L):
    kind, b, ci, h, w, co, k, pad, s = L
    if kind == "linear":
        return 2 * b * ci * co
    return 2 * b * co * _conv_out(h, k, pad, s) * _conv_out(w, k, pad, s) * ci * k * k


def gemm_cpu_reference(workload):
    """The reference's own CPU code (oracle/_ref, OpenMP on all cores) on a bounded sample."""
    from oracle.cpu import Reference
    cores = _omp_all_cores()
    rc = Reference("cnn")
    rng = np.random.default_rng(SEED)
    if workload == "sgemm_4096":
        n = 2048
        A = rng.uniform(-1, 1, n * n).astype(np.float32)
        B = rng.uniform(-1, 1, n * n).astype(np.float32)
        C = np.zeros(n * n, np.float32)
        ts = []
        for _ in range(2):
            t0 = time.perf_counter()
            rc.sgemm("N", "N", n, n, n, 1.0, A, B, 0.0, C)
            ts.append(time.perf_counter() - t0)
        return {"value": 2 * n ** 3 / min(ts) / 1e9, "unit": "GFLOP/s", "cores": cores, "kind": "reference",
                "sample": f"gemm_rnn {n}^3 (17.2 GFLOP), best of 2"}
    # CNN: every layer at batch 4 (the linear layers at 128), scaled to batch 128
    t_total = 0.0
    for L in CNN_LAYERS:
        kind, b, ci, h, w, co, k, pad, s = L
        if kind == "conv":
            bs = 4
            x = rng.uniform(0, 1, bs * ci * h * w).astype(np.float32)
            wt = rng.standard_normal(co * ci * k * k).astype(np.float32)
            t0 = time.perf_counter()
            rc.conv2d_forward(x, wt, bs, ci, h, w, co, k, pad, s)
            t_total += (time.perf_counter() - t0) * b / bs
        else:
            x = rng.uniform(-1, 1, b * ci).astype(np.float32)
            wt = rng.uniform(-1, 1, ci * co + co).astype(np.float32)
            t0 = time.perf_counter()
            rc.linear_forward(x, wt, b, ci, co)
            t_total += time.perf_counter() - t0
    gf = sum(layer_flops(L) for L in CNN_LAYERS)
    return {"value": gf / t_total / 1e9, "unit": "GFLOP/s", "cores": cores, "kind": "reference",
            "sample": f"convolutions at batch 4 scaled x32, linear layers at batch 128; {t_total:.2f} s per forward"}


def run_gemm(args, dist, rank, ws, local):
    """One step: a 4096^3 NN sgemm, or the CNN's conv/linear layers at batch 128."""
    import torch
    from catseye_b200 import _lib
    from catseye_b200 import matmul as mm
    _lib.init(local)
    torch.cuda.set_device(local)
    # a stream of our own: the default stream's handle is 0, which the
    # library reads as "the library's stream" (events there would not see it)
    stream = torch.cuda.Stream()
    sp = stream.cuda_stream
    assert sp != 0
    g = torch.Generator(device="cuda").manual_seed(SEED + rank)

    def urand(n, lo=-1.0, hi=1.0):
        return torch.rand(n, device="cuda", generator=g) * (hi - lo) + lo

    if args.workload == "sgemm_4096":
        n = SGEMM_SIZE
        A, B, Cm = urand(n * n), urand(n * n), torch.empty(n * n, device="cuda")
        flops, launches = 2 * n ** 3, 1
        hA, hB, hC = A.cpu().numpy(), B.cpu().numpy(), np.empty(n * n, np.float32)

        def step():
            mm.sgemm_dev("N", "N", n, n, n, 1.0, A, n, B, n, 0.0, Cm, n, stream=sp)

        def host_step():
            mm.sgemm("N", "N", n, n, n, 1.0, hA, hB, 0.0, hC)
            return hC

        h2d, d2h = 2 * n * n * 4, n * n * 4
        cfg = {"workload": "sgemm_4096", "M": n, "N": n, "K": n, "form": "NN", "alpha": 1.0, "beta": 0.0,
               "l2": "A, B, C 64 MB each (192 MB > 126 MB L2); no flush"}
    else:
        bufs, host = [], []
        for L in CNN_LAYERS:
            kind, b, ci, h, w, co, k, pad, s = L
            if kind == "conv":
                nz = b * co * _conv_out(h, k, pad, s) * _conv_out(w, k, pad, s)
                x, wt = urand(b * ci * h * w, 0.0, 1.0), urand(co * ci * k * k) * (2.0 / (ci * k * k)) ** 0.5
            else:
                nz = b * co
                x, wt = urand(b * ci), urand(ci * co + co) * 0.05
            bufs.append((L, x, wt, torch.empty(nz, device="cuda")))
            host.append((L, x.cpu().numpy(), wt.cpu().numpy()))
        flops = sum(layer_flops(L) for L in CNN_LAYERS)
        launches = 9   # 4 convolutions; per linear layer a bias fill and the GEMM (+ split-K reduce for 8192->256)

        def step():
            for L, x, wt, z in bufs:
                kind, b, ci, h, w, co, k, pad, s = L
                if kind == "conv":
                    mm.conv2d_forward_dev(x, wt, z, b, ci, h, w, co, k, pad, s, stream=sp)
                else:
                    mm.linear_forward_dev(x, wt, z, b, ci, co, stream=sp)

        def host_step():
            out = None
            for L, x, wt in host:
                kind, b, ci, h, w, co, k, pad, s = L
                out = (mm.conv2d_forward(x, wt, b, ci, h, w, co, k, pad, s) if kind == "conv"
                       else mm.linear_forward(x, wt, b, ci, co))
            return out

        h2d = sum(x.nbytes + wt.nbytes for _, x, wt in host)
        d2h = sum(z.numel() * 4 for _, _, _, z in bufs)
        cfg = {"workload": "cnn_forward_b128", "batch": 128, "input": "32x32x3",
               "layers": "conv3x3 3->64, 64->64 (32x32), 64->128, 128->128 (16x16), linear 8192->256, 256->10",
               "excluded": "ReLU and max-pool (elementwise, outside the GEMM path); each layer gets its own input",
               "l2": "activations 32-268 MB per layer; no flush"}

    def barrier():
        if dist:
            dist.barrier()

    torch.cuda.synchronize()   # inputs were made on the default stream
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(local) as clk:
        e0.record(stream)
        for _ in range(args.steps):
            step()
        e1.record(stream)
        e1.synchronize()
    torch.cuda.synchronize()
    barrier()
    ms = e0.elapsed_time(e1)
    if dist:
        t = torch.tensor([ms], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    # end to end through the host-pointer API (copies in and out every step)
    host_step()
    e2e_steps = max(1, min(args.e2e_steps, 3))
    t0 = time.perf_counter()
    for _ in range(e2e_steps):
        host_step()
    e2e_s = time.perf_counter() - t0
    if dist:
        t = torch.tensor([e2e_s], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_s = float(t.item())
    return ms, e2e_s, e2e_steps, flops, launches, h2d, d2h, cfg, clk.summary()


def gemm_main(args):
    metric = "SGEMM GFLOP/s" if args.workload == "sgemm_4096" else "CNN forward GFLOP/s (conv + linear, batch 128)"
    if args.impl == "reference":
        if int(os.environ.get("RANK", "0")) != 0:
            return
        cb = gemm_cpu_reference(args.workload)
        print(json.dumps({"impl": "reference", "metric": metric, "value": round(cb["value"], 2), "unit": "GFLOP/s",
                          "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "higher_is_better": True,
                          "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
                          "config": {"workload": args.workload}, "cpu_baseline": cb,
                          "e2e": {"value": round(cb["value"], 2), "unit": "GFLOP/s", "h2d_bytes_per_step": 0,
                                  "d2h_bytes_per_step": 0}}))
        return
    dist, rank, ws, local = dist_init()
    ms, e2e_s, e2e_steps, flops, launches, h2d, d2h, cfg, clocks = run_gemm(args, dist, rank, ws, local)
    if rank == 0:
        gfs = ws * flops * args.steps / (ms * 1e-3) / 1e9
        achieved = flops * args.steps / (ms * 1e-3) / 1e12
        cfg["parallelism"] = f"replicas{ws}" if ws > 1 else "single"
        # 3xTF32 on tcgen05: three tf32 products per fp32 product, tf32 at half the bf16 rate
        bf16, bf16_kind = tensor_peak()
        peak = bf16 / 2 / 3
        roof = {"bound": "tensor", "peak_kind": f"{bf16_kind} / 2 (tf32 rate) / 3 (products per fp32 product)",
                "kernel": "k_sgemm_tc (3xTF32, tcgen05 kind::tf32)" if args.workload == "sgemm_4096"
                else "k_sgemm_tc conv mode (3 of 4 convolutions) + k_conv_fwd (3->64) + k_sgemm(_tc) (linear)"}
        line = {"metric": metric, "value": round(gfs, 1), "unit": "GFLOP/s", "n_gpus": ws, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 4), "higher_is_better": True,
                "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic", "config": cfg,
                "roofline": dict(roof, achieved=round(achieved, 2), peak=round(peak, 1), unit="TFLOP/s",
                                 frac=round(achieved / peak, 4), traffic=None),
                "e2e": {"value": round(ws * flops * e2e_steps / e2e_s / 1e9, 1), "unit": "GFLOP/s",
                        "h2d_bytes_per_step": int(h2d), "d2h_bytes_per_step": int(d2h)},
                "gpu_launches": launches * args.steps, "clocks": clocks}
        if not args.no_cpu_baseline:
            line["cpu_baseline"] = gemm_cpu_reference(args.workload)
        print(json.dumps(line))
    if dist:
        dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=128)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--e2e-steps", type=int, default=32)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="llama7b_q4_0",
                    choices=sorted(WORKLOADS) + sorted(BATCHED) + ["sgemm_4096", "cnn_forward_b128"])
    ap.add_argument("--layers", type=int, default=0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--replicas", action="store_true",
                    help="decode workloads under torchrun: every rank decodes its own replica instead of one "
                         "model sharded over the ranks by tensor parallelism (the default)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.workload in ("sgemm_4096", "cnn_forward_b128"):
        gemm_main(args)
        return
    if args.workload in BATCHED:
        batched_main(args)
        return

    if args.impl == "reference":
        rank = int(os.environ.get("RANK", "0"))
        if rank != 0:
            return
        ws = int(os.environ.get("WORLD_SIZE", "1"))
        cfg = cfg_for(args.workload, args.layers)
        cb = cpu_reference(cfg, "reference")
        line = {"impl": "reference", "metric": "decode tok/s (batch 1)", "value": round(cb["value"], 3),
                "unit": "tok/s", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
                "ms_per_step": round(1e3 / cb["value"], 3), "higher_is_better": True,
                "scaling": "strong" if ws > 1 and not args.replicas else "weak",
                "vs_baseline": vs_published(args, cb["value"]),
                "dtype": {0: "f32", 2: "q4_0 x q8 (int8 dot, f32 accumulate)",
                                               8: "q8_0 x q8"}[cfg.wtype],
                "data": "synthetic", "config": decode_config(args, cfg, ws, ws > 1 and not args.replicas),
                "cpu_baseline": cb,
                "e2e": {"value": round(cb["value"], 3), "unit": "tok/s", "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}}
        if line["vs_baseline"] is not None:
            line["vs_baseline_of"] = {"value": PUBLISHED[args.workload][0], "unit": "tok/s",
                                      "source": PUBLISHED[args.workload][1]}
        print(json.dumps(line))
        return

    tp_default = int(os.environ.get("WORLD_SIZE", "1")) > 1 and not args.replicas
    dist, rank, ws, local = dist_init("gloo" if tp_default else "nccl")
    r = run_ours(args, dist, rank, ws, local)
    if rank != 0:
        if dist:
            dist.destroy_process_group()
        return
    cfg, ms, tp = r["cfg"], r["ms"], r["tp"]
    peak, peak_kind = peaks()
    seqs = 1 if tp else ws   # sequences decoded by the whole job
    tok_s = seqs * args.steps / (ms * 1e-3)
    achieved = r["kbytes"] / (ms * 1e-3) / 1e9
    if tp and r["engine"] == "persistent":
        kern = "k_decode per GPU with the partial rows of wo and w2 pushed to every peer (%d steps per launch)" % args.steps
    elif tp:
        kern = ("graph engine per GPU: k_matvec / k_attention / residual adds, NCCL allreduce after wo and w2, one "
                "CUDA graph per token")
    else:
        kern = "k_decode (persistent cooperative decode, %d steps per launch)" % args.steps
    line = {
        "metric": "decode tok/s (batch 1)", "value": round(tok_s, 2), "unit": "tok/s", "n_gpus": ws,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 4),
        "higher_is_better": True, "scaling": "strong" if tp else "weak", "vs_baseline": vs_published(args, tok_s),
        "dtype": {0: "f32", 2: "q4_0 x q8 (int8 dot, f32 accumulate)", 8: "q8_0 x q8"}[cfg.wtype],
        "data": "synthetic",
        "config": decode_config(args, cfg, ws, tp),
        "roofline": {"bound": "hbm", "kernel": kern,
                     "achieved": round(achieved, 1), "peak": peak, "peak_kind": peak_kind,
                     "unit": "GB/s", "frac": round(achieved / peak, 4),
                     # DRAM bytes come from ncu captures, which a timed run does not take
                     "traffic": None,
                     "bytes_per_launch": int(r["kbytes"]), "weight_bytes_per_step": int(r["wbytes"]),
                     "ms_per_launch": round(ms, 3)},
        "e2e": {"value": round(seqs * args.e2e_steps / r["e2e_s"], 2), "unit": "tok/s", "h2d_bytes_per_step": 16,
                "d2h_bytes_per_step": cfg.vocab * 4},
        # persistent kernel: one launch (per GPU); graph engine with tensor parallelism: per layer the
        # qkv, attention, wo, w1/w3 and w2 kernels and two residual adds, then the classifier and the
        # advance kernel, per step (the NCCL collectives are NCCL's kernels)
        "gpu_launches": args.steps * (7 * cfg.n_layers + 2) if (tp and r["engine"] == "graph") else 1,
        "clocks": r["clocks"],
    }
    if r["kinds"]:
        line["graph_engine_kernels"] = r["kinds"]
    if r["parity"]:
        line["parity"] = r["parity"]
    if not args.no_cpu_baseline and ws == 1:
        line["cpu_baseline"] = cpu_reference(cfg, "reference")
    if line["vs_baseline"] is not None:
        line["vs_baseline_of"] = {"value": PUBLISHED[args.workload][0], "unit": "tok/s",
                                  "source": PUBLISHED[args.workload][1]}
    print(json.dumps(line))
    if dist:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
