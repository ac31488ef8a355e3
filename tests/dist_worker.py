"""torchrun worker for tests/test_gpu_multi.py: one rank per GPU.

Each rank compiles the 252-step Asian tape on its GPU, joins the engine's
NCCL communicator (unique id broadcast over torch.distributed), replays its
shard of the range with nt_replay_sharded and checks the all-reduced sums
against a single-GPU replay of the whole range on the same device.
"""
import json
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)


def main():
    import datetime

    import numpy as np
    import torch
    import torch.distributed as dist
    from nablatensor_b200 import quant
    from nablatensor_b200.engine import AadOptions, CudaAadEngine, PrecisionEnum, dist_unique_id

    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=60))
    tape = quant.asian_tape(252)
    ex = CudaAadEngine(local).compile(tape, AadOptions(precision=PrecisionEnum.FLOAT64))
    uid = [dist_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(uid, src=0)
    ex.distAttach(world, rank, uid[0], timeout_ms=60_000)
    out = {}
    for total, offset, chunk in [(2_000_000, 0, 0), (10_000_001, 0x1_0000_0003, 1 << 21)]:
        sharded = ex.replaySharded(total, offset, 42, chunk_paths=chunk)
        single = ex.replay(total, offset, 42)
        out[f"{total}"] = {
            "value": [sharded.value(), single.value()],
            "grad_rel": float(np.max(np.abs(sharded.gradients() - single.gradients()) / np.abs(single.gradients()))),
            "value_rel": abs(sharded.value() - single.value()) / abs(single.value()),
        }
    ex.distDetach()
    ex.close()
    dist.barrier()
    dist.destroy_process_group()
    if rank == 0:
        print("RESULT " + json.dumps(out), flush=True)


if __name__ == "__main__":
    main()
