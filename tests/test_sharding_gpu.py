"""sharding.sharded_attention on GPUs (needs a B200; the two-rank test needs two of them).

One GPU, no process group: the call computes the whole problem and must equal the native
operator bit for bit. Two GPUs: two NCCL ranks (127.0.0.1 rendezvous, no multicast anywhere),
each computing its shard - prefill by (batch x head) rows, decode by batch rows balanced by
visible keys - and all-gathering O and LSE; every rank's gathered result must equal the
single-GPU call bit for bit. The shapes are chosen so that the whole call and the shards take
the same kernel configuration (no KV split, the same decode kernel), which makes every row's
arithmetic identical.
"""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

import __graft_entry__

__graft_entry__.import_package()

pytestmark = pytest.mark.gpu


def _needs_gpus(n):
    if not torch.cuda.is_available() or torch.cuda.get_device_capability()[0] != 10:
        pytest.skip("needs an sm_100 GPU")
    if torch.cuda.device_count() < n:
        pytest.skip(f"needs {n} GPUs")


def _inputs(kind, device):
    g = torch.Generator(device="cpu").manual_seed(17)
    if kind == "prefill":
        shape_q = shape_kv = (4, 32, 512, 64)
        past = 0
    else:
        shape_q, shape_kv = (8, 4, 1, 64), (8, 4, 1000, 64)
        past = 999
    q = torch.randn(shape_q, generator=g).to(torch.bfloat16).to(device)
    k = torch.randn(shape_kv, generator=g).to(torch.bfloat16).to(device)
    v = torch.randn(shape_kv, generator=g).to(torch.bfloat16).to(device)
    lens = None
    if kind == "decode":
        lens = torch.randint(1, 1001, (8,), generator=g, dtype=torch.int32).to(device)
    return q, k, v, past, lens


@pytest.mark.parametrize("kind", ["prefill", "decode"])
@torch.no_grad()
def test_sharded_attention_one_gpu_equals_operator(kind):
    _needs_gpus(1)
    from tiny_transformer_b200.operators._extension import load_attention_extension
    from tiny_transformer_b200.sharding import sharded_attention
    q, k, v, past, lens = _inputs(kind, "cuda")
    o, lse = sharded_attention(q, k, v, past, lens, gather=True)
    ref_o, ref_lse = load_attention_extension().attention_forward(q, k, v, past, None, lens)
    assert torch.equal(o, ref_o) and torch.equal(lse, ref_lse)


def _rank(rank, world, port, results):
    import datetime

    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        __graft_entry__.import_package()
        from tiny_transformer_b200.operators._extension import load_attention_extension
        from tiny_transformer_b200.sharding import sharded_attention
        ok = []
        with torch.no_grad():
            for kind in ("prefill", "decode"):
                q, k, v, past, lens = _inputs(kind, f"cuda:{rank}")
                o, lse = sharded_attention(q, k, v, past, lens, gather=True)
                ref_o, ref_lse = load_attention_extension().attention_forward(q, k, v, past, None,
                                                                              lens)
                ok.append(bool(torch.equal(o, ref_o) and torch.equal(lse, ref_lse)))
        results[rank] = ok
    finally:
        dist.destroy_process_group()


def test_sharded_attention_two_gpus_gathers_bitwise():
    _needs_gpus(2)
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    manager = ctx.Manager()
    results = manager.dict()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, results)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
    for p in procs:
        if p.is_alive():
            p.terminate()
            p.join()
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    assert dict(results) == {0: [True, True], 1: [True, True]}
