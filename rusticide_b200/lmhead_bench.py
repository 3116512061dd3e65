"""Times the LM-head paths on one GPU: rsc_lmhead_sample (the GEMM with the
sampler fused into its epilogue), rsc_lmhead_logits + rsc_sample, and the
cuBLAS bf16 GEMM (torch.matmul) + rsc_sample, for a Qwen2.5-sized head
(vocab 151936, dim 4096, bf16 weights) at T 0.8, top-k 40, top-p 0.95.

    python -m rusticide_b200.lmhead_bench [--rows 1 16 64 256 1024] [--calls 20]

Under torch.distributed.run (WORLD_SIZE > 1, one process per GPU) it times the
tensor-parallel form instead: every rank holds its vocabulary rows of W and
runs VocabShardedSampler.sample_lmhead (rsc_lmhead_partial, an NCCL all-gather
of the shard records, rsc_shard_merge); rank 0 prints the max over ranks.

Weights and hidden states are seeded random tensors on the device (no
checkpoint is read). Times are CUDA events over `calls` back-to-back calls
after 3 warm-up calls; one line per batch size.
"""

import argparse

import torch

from rusticide_b200 import SamplingParams, engine


def _time(fn, calls: int) -> float:
    for _ in range(3):
        fn()
    torch.cuda.synchronize()
    a = torch.cuda.Event(enable_timing=True)
    b = torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(calls):
        fn()
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) / calls * 1000.0


def tensor_parallel(args) -> None:
    import os
    from datetime import timedelta

    import torch.distributed as dist

    from rusticide_b200.sharding import VocabShardedSampler

    rank = int(os.environ["RANK"])
    world = int(os.environ["WORLD_SIZE"])
    dev = torch.device("cuda", int(os.environ.get("LOCAL_RANK", rank)))
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", timeout=timedelta(seconds=60), device_id=dev)
    try:
        eng = engine(dev.index)
        vs = VocabShardedSampler(eng, args.vocab)
        g = torch.Generator(device=dev).manual_seed(1 + rank)
        w = (torch.randn(vs.width, args.dim, device=dev, generator=g) * (3.0 / args.dim ** 0.5)).bfloat16()
        params = SamplingParams(0.8, 40, 0.95)
        for rows in args.rows:
            gh = torch.Generator(device=dev).manual_seed(7)  # the same hidden states on every rank
            h = torch.randn(rows, args.dim, device=dev, generator=gh).bfloat16()
            u = torch.rand(rows, device=dev, generator=gh)
            eng.ensure(rows, args.vocab)
            outs = eng._outputs(rows, True)
            t = torch.tensor([_time(lambda: vs.sample_lmhead(h, w, params, uniforms=u, out=outs),
                                    args.calls)], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            if rank == 0:
                print(f"rows={rows} x{world} GPUs: tensor-parallel fused {t.item():.1f} us "
                      f"(max over ranks; {vs.width} vocabulary rows of W per rank)", flush=True)
    finally:
        dist.destroy_process_group()


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--rows", type=int, nargs="+", default=[1, 16, 64, 256, 1024])
    ap.add_argument("--vocab", type=int, default=151936)
    ap.add_argument("--dim", type=int, default=4096)
    ap.add_argument("--calls", type=int, default=20)
    ap.add_argument("--fused-only", action="store_true",
                    help="run only rsc_lmhead_sample (for a profiler capture)")
    args = ap.parse_args()
    import os
    if int(os.environ.get("WORLD_SIZE", "1")) > 1:
        tensor_parallel(args)
        return
    dev = torch.device("cuda", 0)
    eng = engine(0)
    g = torch.Generator(device=dev).manual_seed(1)
    w = (torch.randn(args.vocab, args.dim, device=dev, generator=g) * (3.0 / args.dim ** 0.5)).bfloat16()
    params = SamplingParams(0.8, 40, 0.95)
    for rows in args.rows:
        h = torch.randn(rows, args.dim, device=dev, generator=g).bfloat16()
        u = torch.rand(rows, device=dev, generator=g)
        eng.ensure(rows, args.vocab)
        outs = eng._outputs(rows, True)
        fused = _time(lambda: eng.lmhead_sample(h, w, params, uniforms=u, out=outs), args.calls)
        flops = 2.0 * rows * args.dim * args.vocab
        line = (f"rows={rows}: fused {fused:.1f} us ({flops / fused / 1e6:.0f} TFLOP/s, "
                f"weights {args.vocab * args.dim * 2 / fused / 1e3:.0f} GB/s)")
        if not args.fused_only:
            t_logits = _time(lambda: eng.lmhead_logits(h, w), args.calls)
            logits = eng.lmhead_logits(h, w)
            t_sample = _time(lambda: eng.sample(logits, params, uniforms=u, out=outs), args.calls)
            t_cublas = _time(lambda: torch.matmul(h, w.T), args.calls)
            line += (f" | rsc_lmhead_logits {t_logits:.1f} + rsc_sample {t_sample:.1f}"
                     f" | cuBLAS bf16 {t_cublas:.1f} + rsc_sample {t_sample:.1f}")
        print(line, flush=True)


if __name__ == "__main__":
    main()
