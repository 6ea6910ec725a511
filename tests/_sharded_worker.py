"""torchrun worker for tests/test_gpu_sharded.py: sharded reductions over
the ranks' GPUs, results written by rank 0 as JSON to argv[1]."""
import json
import os
import sys
from datetime import timedelta
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))

import torch
import torch.distributed as dist

import flight4s_b200 as f4s
from flight4s_b200.sharded import ORDERED_GRANULE, ShardedReducer


def main() -> None:
    out_path = sys.argv[1]
    n_total = int(sys.argv[2])
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=120))
    ctx = f4s.CudaContext.open(local)
    hp = ctx.hotpath()
    red = ShardedReducer(hp, dev, n_total)
    x = torch.empty(max(red.count, 1), dtype=torch.float32, device=dev)
    xi = torch.empty(max(red.count, 1), dtype=torch.int32, device=dev)
    hp.fill_synthetic(x, red.count, f4s.UNIFORM_F32, seed=99, offset=red.offset)
    hp.fill_synthetic(xi, red.count, f4s.UNIFORM_I32, seed=99, offset=red.offset, ilo=-1000, ihi=1000)
    xs, xis = x[:red.count], xi[:red.count]
    results = []
    for _ in range(2):  # twice: workspaces and outputs are reused
        red.sum_f32_async(xs)  # three collectives in flight at once
        red.sum_i32_async(xis)
        red.argmax_f32_async(xs)
        red.wait()
        s, i, packed = float(red.f64.item()), int(red.i32.item()), int(red.arg[0].item())
        assert red.sum_i32(xis) == i and red.argmax_f32(xs)[1] >= 0 and red.sum_f32(xs) == s
        # typed sums over inputs derived from the i32 data (same derivation in the test)
        e4m3 = (xis & 0x7E).to(torch.uint8)
        f16 = (xis & 0x3BFF).to(torch.int16).view(torch.float16)
        red.sum_async("u32", xis)
        red.sum_async("e4m3", e4m3)
        red.sum_async("f16", f16)
        red.wait()
        typed = {k: red.sum(k, v) for k, v in (("u32", xis), ("e4m3", e4m3), ("f16", f16))}
        f64 = xs.to(torch.float64)
        for k, v in (("u32", xis.view(torch.int32)), ("f16", f16), ("f64", f64)):
            red.argmax_async(k, v)
        red.wait()
        typed.update({f"argmax_{k}": list(red.argmax(k, v))
                      for k, v in (("u32", xis.view(torch.int32)), ("f16", f16), ("f64", f64))})
        results.append({"sum_f32": s, "sum_i32": i, "argmax_packed": packed, "typed": typed})
    # batched steps with launch overlap (two batches in flight, partials
    # alternating between two buffers): the same results as the plain calls
    hp.set_launch_overlap(True)
    batched = []
    stream = torch.cuda.current_stream()
    for _ in range(2):
        held = []
        for _ in range(2):
            with red.batch(stream):
                red.sum_f32_async(xs, stream)
                red.argmax_f32_async(xs, stream)
                red.sum_i32_async(xis, stream)
            held.append((red.f64, red.i32, red.arg))
        red.wait(stream)
        batched += [[float(b[0].item()), int(b[1].item()), int(b[2][0].item())] for b in held]
    hp.set_launch_overlap(False)
    # order-fixed sums over granule-aligned shards: the same bits as one GPU
    red_o = ShardedReducer(hp, dev, n_total, granule=ORDERED_GRANULE)
    xo = torch.empty(max(red_o.count, 1), dtype=torch.float32, device=dev)
    hp.fill_synthetic(xo, red_o.count, f4s.UNIFORM_F32, seed=99, offset=red_o.offset)
    xos = xo[:red_o.count]
    xob = xos.to(torch.bfloat16)
    ordered = []
    for _ in range(2):
        ordered.append({"f32": red_o.sum("f32", xos, policy="deterministic"),
                        "bf16": red_o.sum("bf16", xob, policy="strict")})
    torch.cuda.synchronize()
    dist.barrier(device_ids=[local])
    if dist.get_rank() == 0:
        Path(out_path).write_text(json.dumps({"world": dist.get_world_size(), "results": results,
                                              "ordered": ordered, "batched": batched}))
    ctx.close()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
