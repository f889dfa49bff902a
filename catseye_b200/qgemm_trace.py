"""Per-K-slice timeline of one batched product on the tensor cores.

    python -m catseye_b200.qgemm_trace [--n 4096] [--d 22016] [--T 16] [--slices 24] [--reps 3]

Builds a random Q4_0 weight of d rows x n columns (the default is the 7B
interleaved w1/w3 product), registers it, and runs the product on random
activations of T tokens.  Prints the plan the library takes (token tile, K
splits, CTAs resident per SM, tensor-map-fed, K slices per split), the time
of the whole product (CUDA events), and CTA (0, 0, 0)'s timeline: for each of
its first K slices, when (µs from the CTA's start, at the SM clock read after
the run) the raw weight copy was issued (a group's first slice), producer
warp 0 got past the raw stage's wait (no later than the copy landed, or
when the producers reached the group), the fp16 stage was free, the last
producer warp was done, the MMA thread found the operands ready and issued
its commit.  Then the mean interval between consecutive stamped slices of
each event, which is the per-slice cost the product pays.
"""
import argparse

import numpy as np


def random_q4_0(n, d, seed):
    """d rows of n/32 Q4_0 blocks: an fp16 scale, then 16 bytes of nibbles."""
    rng = np.random.default_rng(seed)
    nb = n // 32
    blk = np.zeros((d, nb, 18), np.uint8)
    scale = (rng.uniform(0.5, 1.5, (d, nb)) * 2e-3).astype(np.float16)
    blk[:, :, 0:2] = scale.view(np.uint8).reshape(d, nb, 2)
    blk[:, :, 2:] = rng.integers(0, 256, (d, nb, 16), dtype=np.uint8)
    return blk.reshape(-1)


def sm_clock_mhz(dev=0):
    try:
        import pynvml
        pynvml.nvmlInit()
        h = pynvml.nvmlDeviceGetHandleByIndex(dev)
        return float(pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM))
    except Exception:
        return 1965.0


EVENTS = [("raw issued", 0), ("raw reached", 2), ("stage free", 3), ("producers done", None),
          ("operands ready", 12), ("commit", 13)]


def main():
    import torch
    from catseye_b200 import _lib, matmul
    ap = argparse.ArgumentParser()
    ap.add_argument("--n", type=int, default=4096)
    ap.add_argument("--d", type=int, default=22016)
    ap.add_argument("--T", type=int, default=16)
    ap.add_argument("--slices", type=int, default=24)
    ap.add_argument("--reps", type=int, default=3)
    args = ap.parse_args()
    _lib.init(0)
    torch.cuda.set_device(0)
    w = random_q4_0(args.n, args.d, 7)
    matmul.register_weight(w, 2, args.n, args.d)
    x = torch.randn(args.T, args.n, device="cuda")
    y = torch.empty(args.T, args.d, device="cuda")
    torch.cuda.synchronize()
    plan = matmul.qgemm_plan(w, args.T)
    print("plan: token tile %d, K splits %d, resident %d per SM, tensor-map fed %d, %d K slices per split "
          "(occupancy query now: %d, error %d)" % plan)
    # whole-product time on torch's stream
    for _ in range(2):
        matmul.qgemm_dev(w, x, y, args.T, torch.cuda.current_stream().cuda_stream)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(10):
        matmul.qgemm_dev(w, x, y, args.T, torch.cuda.current_stream().cuda_stream)
    e1.record()
    e1.synchronize()
    us = e0.elapsed_time(e1) * 100.0
    wbytes = args.d * args.n // 32 * 18
    print("product: %.2f us, %.1f GB/s of weights" % (us, wbytes / (us * 1e-6) / 1e9))
    slices = min(args.slices, plan[4])
    for rep in range(args.reps):
        tr = matmul.qgemm_trace(w, x, y, args.T, slices).astype(np.int64)
        mhz = sm_clock_mhz()
        t0 = tr[slices, 0]

        def at(v):
            return (v - t0) / mhz if v else float("nan")

        print(f"rep {rep}: SM clock {mhz:.0f} MHz; CTA done at {at(tr[slices, 2]):.2f} us "
              f"(last MMA seen complete {at(tr[slices, 1]):.2f})")
        if rep:
            continue
        print("  slice " + "".join(f"{name:>16s}" for name, _ in EVENTS))
        cols = {}
        for k in range(slices):
            row = []
            for name, e in EVENTS:
                v = tr[k, 4:12].max() if e is None else tr[k, e]
                row.append(at(v))
                cols.setdefault(name, []).append(at(v))
            print(f"  {k:5d} " + "".join(f"{v:16.3f}" for v in row))
        def mean_step(v):
            k = np.flatnonzero(~np.isnan(np.array(v)))   # the stamped slices (raw copies: every fourth)
            return float(np.mean(np.diff(np.array(v)[k]) / np.diff(k))) if len(k) > 1 else float("nan")

        print("  mean interval per slice (us): " + ", ".join(
            f"{name} {mean_step(v):.3f}" for name, v in cols.items()))
    matmul.unregister_weight(w)


if __name__ == "__main__":
    main()
