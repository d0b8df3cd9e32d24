"""Rank program of the two-rank sharding test (launched by torch.distributed.run from test_shard_gpu.py): every rank
runs asrn_b200.shard.forward on its chunk over NCCL, eager and as a captured ShardedForward (built on zero inputs,
then replayed on the real ones); the chunks are gathered and rank 0 compares them with the unsharded layer."""
import datetime
import os
import sys

import torch
import torch.distributed as dist

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))


def main():
    rank, world = int(os.environ['RANK']), int(os.environ['WORLD_SIZE'])
    torch.cuda.set_device(int(os.environ['LOCAL_RANK']))
    dev = torch.device('cuda', int(os.environ['LOCAL_RANK']))
    dist.init_process_group('nccl', timeout=datetime.timedelta(seconds=60))
    from asrn_b200 import shard
    from test_shard_gpu import _layer_and_inputs
    ok = True
    for half, nb in ((False, 6), (True, 14)):
        layer, E, h, x = _layer_and_inputs(dev, 64, 1, 8192, nb)
        c0, c1 = shard.chunk_bounds(8192, world, rank)
        with torch.no_grad(), torch.autocast('cuda', dtype=torch.bfloat16, enabled=half):
            eager = shard.forward(layer, E[:, c0:c1], h[:, c0:c1], x[:, c0:c1])
            # the same forward captured as a CUDA graph (NCCL collectives inside), replayed twice
            sf = shard.ShardedForward(layer, E[:, c0:c1], h[:, c0:c1], x[:, c0:c1])
            sf(E[:, c0:c1], h[:, c0:c1], x[:, c0:c1])
            graphed = sf(E[:, c0:c1], h[:, c0:c1], x[:, c0:c1]).clone()
            torch.cuda.synchronize()
            shard.check_exchange(dev)
            sf.close()
            # built on inputs whose tails are all in one bucket, the exchange is sized too small for the real ones:
            # a replay on them must be reported, not silently wrong
            small = shard.ShardedForward(layer, torch.zeros_like(E[:, c0:c1]), torch.zeros_like(h[:, c0:c1]),
                                         x[:, c0:c1], margin=1.0, extra=0)
            small(E[:, c0:c1], h[:, c0:c1], x[:, c0:c1])
            torch.cuda.synchronize()
            try:
                shard.check_exchange(dev)
                raised = 0
            except shard.ShardExchangeError:
                raised = 1
            small.close()
            flag_r = torch.tensor([raised], device=dev)
            dist.all_reduce(flag_r, op=dist.ReduceOp.MAX)
            if rank == 0:
                print(f'overflow reported: {bool(flag_r.item())}', flush=True)
            ok = ok and bool(flag_r.item())
            for name, mine in (('eager', eager), ('graph', graphed)):
                parts = [torch.empty_like(mine) for _ in range(world)]
                dist.all_gather(parts, mine.contiguous())
                if rank == 0:
                    ref = layer(E, h, x)
                    got = torch.cat(parts, 1)
                    err = ((got - ref).abs().max() / ref.abs().max()).item()
                    tol = 2e-2 if half else 1e-4
                    print(f'{name} half={half} rel err {err:.3e}', flush=True)
                    ok = ok and err <= tol
    flag = torch.tensor([1 if ok else 0], device=dev)
    dist.broadcast(flag, 0)
    dist.barrier()
    dist.destroy_process_group()
    if rank == 0 and flag.item():
        print('shard ranks ok', flush=True)
    sys.exit(0 if flag.item() else 1)


if __name__ == '__main__':
    main()
