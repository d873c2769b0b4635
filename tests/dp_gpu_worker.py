"""One rank of the 2-GPU data-parallel parity check (run by torchrun from
tests/test_dp_gpu.py): every rank takes its shard of a fixed global batch,
steps the trainer twice, and rank 0 writes the adapter it ends with, the
loss, and whether all ranks hold identical parameters."""
from __future__ import annotations

import datetime
import os
import sys
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parent.parent))


def main() -> int:
    import torch
    import torch.distributed as dist

    from torobi_b200.model import QLoRACausalLM, tiny_config
    from torobi_b200.train import AdamWConfig, NcclGradReduce, Trainer, dist_env, shard_rows

    rank, world, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=120))
    cfg = tiny_config(lora_targets=("q_proj", "v_proj", "down_proj"))
    model = QLoRACausalLM(cfg, dev, seed=11)
    g = torch.Generator(device=dev)
    g.manual_seed(5)
    ids = torch.randint(0, cfg.vocab, (8, 128), generator=g, device=dev)  # same on every rank
    lo, hi = shard_rows(8, world, rank)
    reduce = NcclGradReduce(rank, world, dist.distributed_c10d._get_default_store())
    tr = Trainer(model, AdamWConfig(lr=1e-2), micro_batch=2, reduce=reduce, rank=rank, world=world)
    losses = []
    for _ in range(2):
        losses.append(float(tr.step(ids[lo:hi])))
        tr.settle()
    params = model.store.params.clone()
    gathered = [torch.empty_like(params) for _ in range(world)]
    dist.all_gather(gathered, params)
    same = all(torch.equal(gathered[0], x) for x in gathered)
    if rank == 0:
        out = Path(os.environ["TQ_DP_OUT"])
        torch.save({"params": params.cpu(), "losses": losses, "same": same}, out)
    reduce.close()
    dist.barrier()
    dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
