"""torchrun worker for tests/test_gpu_sharded.py: two ranks run one sharded
step on their GPUs; then rank 1 leaves between steps (announced through
the rank monitor, with nothing of its own in flight) and rank 0 must raise
RankFailure on the host before launching anything of step 2 and abort its
communicator; it reports how long the detection and the abort each took
(JSON to argv[1])."""
import json
import os
import sys
import time
from datetime import timedelta
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))

import torch
import torch.distributed as dist

import flight4s_b200 as f4s
from flight4s_b200.sharded import RankFailure, RankMonitor, ShardedReducer


def main() -> None:
    out_path = sys.argv[1]
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=60))
    ctx = f4s.CudaContext.open(local)
    hp = ctx.hotpath()
    red = ShardedReducer(hp, dev, 1 << 24, monitor=RankMonitor(timeout_s=10.0))
    x = torch.empty(red.count, dtype=torch.float32, device=dev)
    hp.fill_synthetic(x, red.count, f4s.UNIFORM_F32, seed=5, offset=red.offset)
    red.begin_step()
    first = red.sum_f32(x)
    torch.cuda.synchronize()
    if dist.get_rank() == 1:
        red.monitor.leave()  # between steps: nothing of this rank is in flight
        ctx.close()
        dist.destroy_process_group()
        return
    t0 = time.monotonic()
    t_abort = None
    try:
        red.begin_step()
        outcome = "no error"
    except RankFailure:
        outcome = "RankFailure"
        t_abort = time.monotonic()
        red.abort()
    elapsed = (t_abort if t_abort is not None else time.monotonic()) - t0
    abort_s = time.monotonic() - t_abort if t_abort is not None else None
    Path(out_path).write_text(json.dumps({"first": first, "outcome": outcome, "elapsed": elapsed, "abort_s": abort_s}))
    ctx.close()


if __name__ == "__main__":
    main()
