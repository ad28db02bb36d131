"""One rank of the two-GPU sequence-sharded decode test (test infrastructure;
run by test_gpu_split_kv.py through torch.distributed.run).  Every rank
builds the same seeded case on its own GPU, decodes its page range, exchanges
partial blocks over NCCL and merges; the merged output is compared with the
numpy oracle and the check's outcome (0 = pass) is written to RESULT_DIR."""

import os
import sys
from datetime import timedelta

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
for p in (HERE, ROOT, os.path.join(ROOT, "intent-attention-kernel_b200"), os.path.join(HERE, "golden")):
    sys.path.insert(0, p)

import numpy as np  # noqa: E402
import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402


def main():
    rank, local = int(os.environ["RANK"]), int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=60), device_id=dev)
    from gpu_cases import make_case, run_oracle, tag_map_for
    from intent_attention.split_kv import SequenceShardedDecoder, shard_page_lists
    case = make_case(941, B=3, Hq=32, Ht=8, W=150, NP=1800, formats=("F16", "FP8", "INT8", "INT4"), device=dev)
    world = dist.get_world_size()
    lt, lc = shard_page_lists(case["table"], case["counts"], rank, world)
    ref = run_oracle(case)
    ok = True
    for transport in ("nccl", "p2p"):
        dec = SequenceShardedDecoder(transport=transport)
        for _ in range(3):      # both exchange parities and a reuse
            out = dec.decode(case["q"], case["pool"], lt, lc, case["tags"], tag_map_for(case["formats"]),
                             out=torch.empty(case["q"].shape, dtype=torch.float32, device=dev))
        torch.cuda.synchronize(dev)
        if transport == "p2p":
            dec._x.check()
        ok = ok and np.allclose(out.cpu().numpy(), ref, atol=2e-3, rtol=1e-2)
        dist.barrier()
        dec.close()
    np.save(os.path.join(os.environ["RESULT_DIR"], f"rank{rank}.npy"), np.array([0.0 if ok else 1.0]))
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
