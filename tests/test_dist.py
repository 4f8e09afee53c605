"""Multi-rank host logic on CPU with the gloo backend (world size 2):
shard arithmetic, sharded results equal to the unsharded run, and the
max-over-ranks timing reduction bench.py uses."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from conftest import ROOT, load_pkg


def test_shard_bh_partitions_exactly():
    sh = load_pkg().sharding
    for total in (1, 7, 128, 192):
        for world in (1, 2, 3, 4, 8):
            spans = [sh.shard_bh(total, r, world) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == total
            for (a, b), (c, d) in zip(spans, spans[1:]):
                assert b == c
            sizes = [b - a for a, b in spans]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        sh.shard_bh(8, 2, 2)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, out_dir):
    import sys
    sys.path.insert(0, ROOT)
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import torch.distributed as dist
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    import oracle
    pkg = load_pkg()
    sh = pkg.sharding
    inp = pkg.workloads.mixer_inputs(2, 3, 128, 16, 0, 64, seed=5)
    start, end = sh.shard_bh(6, rank, world)
    names = ["q", "k", "v", "alpha", "beta", "mu"]
    local = [sh.slice_heads(getattr(inp, n), start, end) for n in names]
    o = oracle.mixer_core_forward(*local, None, 0, 3, 64)
    torch.save(o, os.path.join(out_dir, f"o{rank}.pt"))
    t = sh.max_over_ranks(float(rank + 1) * 1.5)
    torch.save(t, os.path.join(out_dir, f"t{rank}.pt"))
    dist.barrier()
    dist.destroy_process_group()


def test_two_rank_shards_match_single_run(tmp_path):
    world = 2
    mp.start_processes(_worker, args=(world, _free_port(), str(tmp_path)), nprocs=world,
                       join=True, start_method="spawn")
    import oracle
    pkg = load_pkg()
    inp = pkg.workloads.mixer_inputs(2, 3, 128, 16, 0, 64, seed=5)
    full = oracle.mixer_core_forward(inp.q, inp.k, inp.v, inp.alpha, inp.beta, inp.mu, None,
                                     0, 3, 64).reshape(6, 128, 16)
    parts = [torch.load(tmp_path / f"o{r}.pt")[0] for r in range(world)]
    assert torch.equal(torch.cat(parts, 0), full)
    for r in range(world):
        assert torch.load(tmp_path / f"t{r}.pt") == 3.0
