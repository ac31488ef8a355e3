"""torchrun worker for tests/test_gpu_multi.py: one rank per GPU.

NT_DIST_CASE=parity (the default): each rank compiles the 252-step Asian tape
on its GPU, joins the engine's NCCL communicator (unique id broadcast over
torch.distributed with gloo), replays its shard of the range with
nt_replay_sharded and checks the all-reduced sums
  - against a single-GPU replay of the whole range on the same device: the
    same bits, since shards are whole 32-path tiles summed exactly;
  - on rank 0, against the CPU oracle at the same (total, offset, seed), all
    seven channels, plain relative error.
Cases: 2,000,000 paths at offset 0, and a ragged 2,000,003 at offset
0x1_0000_0003 (the high word of the path counter in play, as in the
reference's CudaCheckpointParityTest) in chunks of 2^19.

NT_DIST_CASE=leave: every rank attaches, then rank 1 leaves (it exits
cleanly, nothing of its own in flight) and rank 0 calls nt_replay_sharded with
a 5 s communicator timeout: it must get NT_E_NCCL within the timeout after its
shard, never hang, and its executable must still replay on its own GPU.
"""
import json
import os
import sys
import time

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)


def parity(ex, tape, rank, dist):
    import numpy as np

    out = {}
    for total, offset, chunk in [(2_000_000, 0, 0), (2_000_003, 0x1_0000_0003, 1 << 19)]:
        sharded, _ = ex.replaySharded_sums(total, offset, 42, chunk)
        single, _ = ex.replay_sums(total, offset, 42)
        case = {"same_bits_as_one_gpu": sharded.tobytes() == single.tobytes(),
                "max_rel_vs_one_gpu": float(np.max(np.abs(sharded - single) / np.abs(single))),
                "price": float(sharded[0] / total)}
        if rank == 0:
            from oracle import oracle as O
            want = O.replay(O.FlatTape.of(tape), [100.0, 100.0, 0.20, 0.03, 1.0], total, offset, 42,
                            threads=os.cpu_count(), exact=True).sums
            case["rel_vs_oracle"] = [float(r) for r in np.abs(sharded - want) / np.abs(want)]
        out[f"{total}@{offset:#x}"] = case
        dist.barrier()
    return out


def leave(ex, rank, dist):
    import numpy as np
    import torch
    from nablatensor_b200 import _lib

    torch.cuda.synchronize()
    dist.barrier()  # every rank is attached and idle
    if rank != 0:
        time.sleep(0.5)
        os._exit(0)  # leaves between steps: no kernel or collective of its own in flight
    time.sleep(3.0)  # let the peer's process end first
    t0 = time.perf_counter()
    code, message = 0, ""
    try:
        ex.replaySharded_sums(2_000_000, 0, 42, 0)
    except _lib.NablaError as e:
        code, message = e.code, str(e)
    elapsed = time.perf_counter() - t0
    # The executable stays usable on its own GPU after the abort.
    alone, _ = ex.replay_sums(100_000, 0, 42)
    return {"code": code, "message": message, "elapsed_s": elapsed,
            "replay_after_abort_finite": bool(np.all(np.isfinite(alone)))}


def main():
    import datetime

    import torch
    import torch.distributed as dist
    from nablatensor_b200 import quant
    from nablatensor_b200.engine import AadOptions, CudaAadEngine, PrecisionEnum, dist_unique_id

    case = os.environ.get("NT_DIST_CASE", "parity")
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=120))
    tape = quant.asian_tape(252)
    ex = CudaAadEngine(local).compile(tape, AadOptions(precision=PrecisionEnum.FLOAT64))
    uid = [dist_unique_id() if rank == 0 else None]
    dist.broadcast_object_list(uid, src=0)
    ex.distAttach(world, rank, uid[0], timeout_ms=5_000 if case == "leave" else 60_000)
    if case == "leave":
        res = leave(ex, rank, dist)
        ex.close()
        print("RESULT " + json.dumps(res), flush=True)
        os._exit(0)  # the peer is gone: no collective teardown
    res = parity(ex, tape, rank, dist)
    ex.distDetach()
    ex.close()
    dist.barrier()
    dist.destroy_process_group()
    if rank == 0:
        print("RESULT " + json.dumps(res), flush=True)


if __name__ == "__main__":
    main()
