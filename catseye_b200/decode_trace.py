"""Phase timeline of one step of the persistent decode kernel.

    python -m catseye_b200.decode_trace [--type 2] [--layers 32] [--pos 8] [--reps 3]
    torchrun --nproc-per-node N -m catseye_b200.decode_trace ...   (tensor parallel, rank 0 prints)

Runs a Llama-2-7B-shaped model (random weights, the given weight type and
layer count), feeds a few prompt tokens, then traces single steps: thread 0
of every CTA stamps %globaltimer and its SM's clock64 at each phase boundary
of the kernel.  A matvec is split into: waiting for its first weight chunk
(`_wait`), the dots (`_dots`, first chunk ready to last dot done) and the
epilogue (`_epi`).  Printed per phase kind, summed over layers: the mean time
a CTA spends in it (from globaltimer, and from clock64 at the step's mean
clock rate), and the critical path (latest CTA to finish the phase minus the
earliest to start it, globaltimer).
"""
import argparse
from dataclasses import replace

import numpy as np


def _mv(name):
    return [f"{name}_wait", f"{name}_dots", f"{name}_epi"]


PHASES = (["stage_qkv"] + _mv("mv_qkv") + ["sync_qkv", "attention", "sync_attn", "stage_wo"] + _mv("mv_wo") +
          ["sync_wo", "stage_w13"] + _mv("mv_w13") + ["sync_w13", "stage_w2"] + _mv("mv_w2") + ["sync_w2"])
TAIL = ["stage_cls"] + _mv("mv_cls") + ["argmax_and_syncs"]


def phase_table(ns, clk, n_layers):
    """{phase: (mean us per CTA from ns, mean us per CTA from clock64, critical us)} summed over layers."""
    ns = ns.astype(np.int64)
    clk = clk.astype(np.int64)
    t = (ns - ns[:, 0].min()) / 1e3
    end = 1 + len(PHASES) * n_layers + len(TAIL) - 1
    mhz = float(np.mean((clk[:, end] - clk[:, 0]) / np.maximum(ns[:, end] - ns[:, 0], 1) * 1e3))
    c = clk / mhz
    out = {}

    def add(name, i):
        m, mc, cr = out.get(name, (0.0, 0.0, 0.0))
        out[name] = (m + float((t[:, i] - t[:, i - 1]).mean()), mc + float((c[:, i] - c[:, i - 1]).mean()),
                     cr + float(t[:, i].max() - t[:, i - 1].min()))

    for l in range(n_layers):
        for k, name in enumerate(PHASES):
            add(name, 1 + len(PHASES) * l + k)
    for k, name in enumerate(TAIL):
        add(name, 1 + len(PHASES) * n_layers + k)
    return out, float(t[:, end].max()), mhz


def main():
    from catseye_b200 import _lib, llm
    ap = argparse.ArgumentParser()
    ap.add_argument("--type", type=int, default=llm.Q4_0)
    ap.add_argument("--layers", type=int, default=32)
    ap.add_argument("--pos", type=int, default=8)
    ap.add_argument("--reps", type=int, default=3)
    ap.add_argument("--model", default="LLAMA2_7B", choices=["LLAMA2_7B", "LLAMA2_70B"])
    args = ap.parse_args()
    import os
    ws, rank = int(os.environ.get("WORLD_SIZE", "1")), int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    _lib.init(local)
    cfg = replace(getattr(llm, args.model).with_type(args.type), n_layers=args.layers)
    dist = None
    if ws > 1:   # every rank traces the same steps of one sharded model
        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("gloo")
        m = llm.GpuLLM(cfg, rank, ws)
        m.tp_connect(llm.tp_share_id())
        assert m.tp_persistent(), "the sharded model did not map its peers"
    else:
        m = llm.GpuLLM(cfg)
    m.init_random(7)
    if dist:
        dist.barrier()
    for pos in range(args.pos):
        m.step(pos + 1, pos)
    per_cta = 1 + len(PHASES) * args.layers + len(TAIL) + 8
    for rep in range(args.reps):
        if dist:
            dist.barrier()
        ns, clk = m.trace_step(5, args.pos + rep, per_cta)
        if rank:
            continue
        tab, total, mhz = phase_table(ns, clk, args.layers)
        print(f"step at pos {args.pos + rep}: {total:.1f} us, SM clock {mhz:.0f} MHz")
        for name, (mean, mean_c, crit) in tab.items():
            per = args.layers if name in PHASES else 1
            print(f"  {name:18s} mean/CTA {mean / per:6.2f} us (clock64 {mean_c / per:6.2f})  "
                  f"critical {crit / per:6.2f} us   [per layer; total {mean:7.1f} us]")
    m.close()
    if dist:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
