"""One rank of the 2-GPU data-parallel check (launched by tests/test_dp_gpu.py through torch.distributed.run).

Each rank trains its half of the training-tiny batch through the library's NCCL-bucketed trainer and one clipped
AdamW step; rank 0 also runs a single-GPU trainer that accumulates both halves at scale 1/2 and steps once.  Writes
rank{r}.npz (parameters after the step, the norm) and, on rank 0, single.npz into the directory given.
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))
sys.path.insert(0, HERE)

MAX_NORM = 0.05


def main(out):
    import datetime
    import torch
    import torch.distributed as dist
    import laya_b200
    from test_train_gpu import desc_for, fixture_items, tiny
    rank, world, local = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"]), int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=60))
    cfg, w, g = tiny()
    items = fixture_items(g)
    coeff = [np.array(it["coeff"], np.float32) for it in g["batch"]["items"]]
    halves = [[0, 1], [2]]
    desc = desc_for(cfg, max_tokens=256, max_items=16, max_markers=64)
    t = laya_b200.Trainer(desc, laya_b200.train_desc(max_segment=128), device=local)
    uid = [laya_b200.Trainer.unique_id() if rank == 0 else None]
    dist.broadcast_object_list(uid, src=0)
    t.comm_init(uid[0], rank, world)
    t.load(w)
    mine = halves[rank]
    b = t.batch([items[i] for i in mine])
    t.forward(b)
    t.backward(b, [coeff[i] for i in mine])
    norm = t.clip_and_step(max_norm=MAX_NORM)
    names = t.names()
    np.savez(os.path.join(out, f"rank{rank}.npz"), norm=norm, **{n: t.download(n, (r, c)) for n, r, c in names})
    if rank == 0:
        s = laya_b200.Trainer(desc, laya_b200.train_desc(max_segment=128), device=local)
        s.load(w)
        for half in halves:
            bh = s.batch([items[i] for i in half])
            s.forward(bh)
            s.backward(bh, [coeff[i] * np.float32(0.5) for i in half])
        sn = s.clip_and_step(max_norm=MAX_NORM)
        np.savez(os.path.join(out, "single.npz"), norm=sn, **{n: s.download(n, (r, c)) for n, r, c in names})
        s.close()
    t.close()
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main(sys.argv[1])
