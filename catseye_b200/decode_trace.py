"""Phase timeline of one step of the persistent decode kernel.

    python -m catseye_b200.decode_trace [--type 2] [--layers 32] [--pos 8] [--reps 3]

Runs a Llama-2-7B-shaped model (random weights, the given weight type and
layer count), feeds a few prompt tokens, then traces single steps: thread 0
of every CTA stamps %globaltimer at each phase boundary of the kernel
(activation staging, each matvec, each grid barrier, attention).  Printed
per phase kind, summed over layers: the mean time a CTA spends in it, and
the critical path (latest CTA to finish the phase minus earliest to start).
"""
import argparse
from dataclasses import replace

import numpy as np

PHASES = ["stage_qkv", "mv_qkv", "sync_qkv", "attention", "sync_attn", "stage_wo", "mv_wo", "sync_wo",
          "stage_w13", "mv_w13", "sync_w13", "stage_w2", "mv_w2", "sync_w2"]


def phase_table(tr, n_layers):
    """Per-phase (mean per CTA, critical path) in microseconds, summed over layers."""
    tr = tr.astype(np.int64)
    t = (tr - tr[:, 0].min()) / 1e3
    out = {}
    for l in range(n_layers):
        b = 1 + len(PHASES) * l
        for k, name in enumerate(PHASES):
            prev, cur = t[:, b + k - 1], t[:, b + k]
            m, c = out.get(name, (0.0, 0.0))
            out[name] = (m + float((cur - prev).mean()), c + float(cur.max() - prev.min()))
    b = 1 + len(PHASES) * n_layers
    for k, name in enumerate(["stage_cls", "mv_cls", "argmax_and_syncs"]):
        prev, cur = t[:, b + k - 1], t[:, b + k]
        out[name] = (float((cur - prev).mean()), float(cur.max() - prev.min()))
    return out, float(t[:, b + 2].max())


def main():
    from catseye_b200 import _lib, llm
    ap = argparse.ArgumentParser()
    ap.add_argument("--type", type=int, default=llm.Q4_0)
    ap.add_argument("--layers", type=int, default=32)
    ap.add_argument("--pos", type=int, default=8)
    ap.add_argument("--reps", type=int, default=3)
    args = ap.parse_args()
    _lib.init(0)
    cfg = replace(llm.LLAMA2_7B.with_type(args.type), n_layers=args.layers)
    m = llm.GpuLLM(cfg)
    m.init_random(7)
    for pos in range(args.pos):
        m.step(pos + 1, pos)
    for rep in range(args.reps):
        tr = m.trace_step(5, args.pos + rep)
        tab, total = phase_table(tr, args.layers)
        print(f"step at pos {args.pos + rep}: {total:.1f} us")
        for name, (mean, crit) in tab.items():
            per = args.layers if name in PHASES else 1
            print(f"  {name:18s} mean/CTA {mean:8.1f} us ({mean / per:6.2f} per layer)  "
                  f"critical {crit:8.1f} us ({crit / per:6.2f} per layer)")
    m.close()


if __name__ == "__main__":
    main()
