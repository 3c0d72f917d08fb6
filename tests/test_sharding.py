"""Multi-GPU sharding logic on CPU: partition functions, and a world-size-2 gloo run of the
shard -> compute -> all_gather path with the CPU oracle standing in for the GPU kernel."""
import os
import socket
import sys

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

# Spawned ranks import this module afresh: make the package importable before using it.
sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
import __graft_entry__  # noqa: E402

__graft_entry__.import_package()
from tiny_transformer_b200.sharding import (Shard, balanced_batch_shards, even_shards,
                                            gather_outputs, run_sharded)


def test_even_shards_cover_and_balance():
    for n, w in ((48, 1), (48, 2), (48, 8), (6, 4), (3, 8), (0, 2)):
        shards = even_shards(n, w)
        assert shards[0].start == 0 and shards[-1].stop == n
        assert all(a.stop == b.start for a, b in zip(shards, shards[1:]))
        sizes = [s.size for s in shards]
        assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        even_shards(4, 0)


def test_balanced_batch_shards():
    rng = np.random.default_rng(2026)
    lens = rng.integers(1024, 8193, size=64).tolist()
    for w in (1, 2, 4, 8):
        shards = balanced_batch_shards(lens, w)
        assert shards[0].start == 0 and shards[-1].stop == 64
        assert all(a.stop == b.start for a, b in zip(shards, shards[1:]))
        assert all(s.size >= 1 for s in shards)
        loads = [sum(lens[s.start:s.stop]) for s in shards]
        # No rank carries more than its even share plus one sequence.
        assert max(loads) <= sum(lens) / w + max(lens)
    assert [s.size for s in balanced_batch_shards([5, 0, 0, 5], 2)] == [2, 2] or \
        sum(s.size for s in balanced_batch_shards([5, 0, 0, 5], 2)) == 4


def _oracle_compute(q, k, v, past_len, kv_lens):
    from oracle import attention_oracle as oracle
    qn, kn, vn = (x.float().numpy() for x in (q, k, v))
    if kv_lens is not None:
        o, lse = oracle.decode_with_kv_lens(qn, kn, vn, kv_lens.numpy())
    else:
        o, lse = oracle.attention_fp64(qn, kn, vn, past_len)
    return torch.from_numpy(o).float(), torch.from_numpy(lse).float()


def _worker(rank, world, port, case, out_q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        g = torch.Generator().manual_seed(7)
        if case == "prefill":
            q, k, v = [torch.randn(2, 3, 20, 64, generator=g).bfloat16() for _ in range(3)]
            past, lens = 0, None
        else:
            q = torch.randn(5, 2, 1, 64, generator=g).bfloat16()
            k, v = [torch.randn(5, 2, 40, 64, generator=g).bfloat16() for _ in range(2)]
            past, lens = 39, torch.tensor([40, 3, 17, 0, 29], dtype=torch.int32)
        o, lse, shard, axis = run_sharded(_oracle_compute, q, k, v, past, rank, world, lens)
        if axis == "bh":
            sizes = [s.size for s in even_shards(q.shape[0] * q.shape[1], world)]
        else:
            sizes = [s.size for s in balanced_batch_shards(lens.tolist(), world)]
        full_o, full_lse = gather_outputs(o, lse, sizes, tuple(q.shape), axis)
        ref_o, ref_lse = _oracle_compute(q, k, v, past, lens)
        ok = torch.equal(full_o, ref_o) and torch.equal(full_lse, ref_lse)
        out_q.put((rank, ok, shard.size))
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("case", ["prefill", "decode"])
def test_gloo_world2_shard_and_gather(case):
    ctx = mp.get_context("spawn")
    out_q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, case, out_q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=180)
        assert p.exitcode == 0
    results = sorted(out_q.get(timeout=10) for _ in range(2))
    assert all(ok for _, ok, _ in results)
    assert sum(size for _, _, size in results) == (6 if case == "prefill" else 5)
