"""torchrun worker for tests/test_gpu_sharded.py: sharded max/argmax over
more than 2^32 elements (global indices past the packed key's 32 bits),
results written by rank 0 as JSON to argv[1]."""
import json
import os
import sys
from datetime import timedelta
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))

import torch
import torch.distributed as dist

import flight4s_b200 as f4s
from flight4s_b200.sharded import ShardedReducer

# global index -> planted value: a smaller maximum on rank 0, two equal
# maxima past 2^32 on rank 1 (the lower index must win)
PLANTED = {7: 500.0, (1 << 32) + 100: 1000.0, (1 << 32) + 50: 1000.0}


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
    assert not red.packed_argmax
    x = torch.empty(red.count, dtype=torch.float32, device=dev)
    hb = torch.empty(red.count, dtype=torch.bfloat16, device=dev)
    hp.fill_synthetic(x, red.count, f4s.NORMAL_F32, seed=5, offset=red.offset, p0=0.0, p1=1.0)
    hp.fill_synthetic(hb, red.count, f4s.NORMAL_BF16, seed=5, offset=red.offset, p0=0.0, p1=1.0)
    for g, v in PLANTED.items():
        if red.offset <= g < red.offset + red.count:
            x[g - red.offset] = v
            hb[g - red.offset] = v
    torch.cuda.synchronize()
    results = []
    for _ in range(2):  # twice: the record buffers are reused
        f32 = red.argmax_f32(x)
        bf16 = red.argmax("bf16", hb.view(torch.int16))
        results.append({"f32": list(f32), "bf16": list(bf16)})
    if dist.get_rank() == 0:
        Path(out_path).write_text(json.dumps({"world": dist.get_world_size(), "results": results}))
    dist.barrier()
    del red
    ctx.close()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
