"""Profiling driver: run a few forwards of one synthetic MoE block, for use under ncu.

    python -m diskmule_b200.prof --config qwen35 --tokens 512 --reps 3

Each forward launches the same kernels as the benchmark (CUDA graphs off, so every
kernel is a separate launch that ncu can select with -k / -s / -c). Prints "ok".
"""
from __future__ import annotations

import argparse
import os


def main() -> None:
    p = argparse.ArgumentParser()
    p.add_argument("--config", default="qwen35")
    p.add_argument("--tokens", type=int, default=512)
    p.add_argument("--reps", type=int, default=3)
    p.add_argument("--seed", type=int, default=1)
    args = p.parse_args()
    os.environ["DISKMULE_CUDA_GRAPHS"] = "0"

    import torch

    from .moe import CudaContext
    from .synthetic import build_layer, input_spec

    ctx = CudaContext(0)
    sl = build_layer(ctx, args.config, seed=args.seed)
    cfg, T = sl.cfg, args.tokens
    xdt = torch.bfloat16 if cfg["family"] == "glm52" else torch.float32
    x = torch.empty((T, cfg["hidden"]), dtype=xdt, device="cuda")
    y = torch.empty((T, cfg["hidden"]), dtype=torch.float32, device="cuda")
    input_spec(cfg, T, 5).device_fill(x.data_ptr())
    ctx.synchronize()
    stream = torch.cuda.current_stream().cuda_stream
    for _ in range(args.reps):
        sl.layer.forward(x.data_ptr(), y.data_ptr(), T, stream=stream)
    torch.cuda.synchronize()
    sl.close()
    print("ok")


if __name__ == "__main__":
    main()
