"""Multi-process (gloo, world_size 2, CPU) checks of the sharding logic used by
multi-GPU runs: each rank computes its (batch or head) shard with the oracle and
the gathered result equals the unsharded computation; a rank that fails is
reported to the others through the process group instead of hanging them."""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from conftest import PKG_DIR, ROOT


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, mode, resq):
    import sys
    sys.path.insert(0, str(ROOT))
    sys.path.insert(0, str(PKG_DIR))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=30))
    try:
        from gdn_b200.sharding import batch_shard, head_shard, slice_heads, gather_shards
        from gdn_b200.synthetic import make_inputs
        from oracle import gdn_oracle as O
        if mode == "batch":
            inp = make_inputs(4, 70, 2, 4, 128, seed=3)
            b0, b1 = batch_shard(4, world, rank)
            o, s = O.chunk_gated_delta_rule(inp.q[b0:b1], inp.k[b0:b1], inp.v[b0:b1], inp.g[b0:b1],
                                            inp.beta[b0:b1], 64, inp.s0[b0:b1])
            o_all = gather_shards(torch.from_numpy(o), world, 0).numpy()
            s_all = gather_shards(torch.from_numpy(s), world, 0).numpy()
        elif mode == "head":
            inp = make_inputs(1, 90, 4, 8, 128, seed=4)
            sh = head_shard(8, 4, world, rank)
            q, k, v, g, b, _, s0 = slice_heads(sh, inp.q, inp.k, inp.v, inp.g, inp.beta, None, inp.s0)
            o, s = O.chunk_gated_delta_rule(q, k, v, g, b, 64, s0)
            o_all = gather_shards(torch.from_numpy(np.ascontiguousarray(o)), world, 2).numpy()
            s_all = gather_shards(torch.from_numpy(s), world, 1).numpy()
        else:  # "fail": rank 1 raises before the collective; rank 0 must get an error, not hang
            if rank == 1:
                raise RuntimeError("injected host-side failure")
            t = torch.zeros(1)
            dist.all_reduce(t)
            resq.put((rank, "no-error"))
            return
        if rank == 0:
            o_ref, s_ref = O.chunk_gated_delta_rule(inp.q, inp.k, inp.v, inp.g, inp.beta, 64, inp.s0)
            resq.put((rank, bool(np.array_equal(o_all, o_ref) and np.allclose(s_all, s_ref, rtol=0, atol=0))))
    except RuntimeError as e:
        resq.put((rank, f"error: {type(e).__name__}"))
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def _run(mode, world=2, timeout=120):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, mode, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = []
    for p in procs:
        p.join(timeout)
        if p.is_alive():
            p.kill()
            p.join()
    while not q.empty():
        results.append(q.get())
    return dict(results)


@pytest.mark.parametrize("mode", ["batch", "head"])
def test_sharded_equals_unsharded(mode):
    res = _run(mode)
    assert res.get(0) is True, res


def test_failed_rank_surfaces_as_error_not_hang():
    res = _run("fail", timeout=90)
    assert res.get(1, "").startswith("error"), res
    assert res.get(0, "").startswith("error"), res


def test_head_shard_mapping():
    from gdn_b200.sharding import head_shard
    # config 3: 32 v-heads, 16 qk-heads over 8 GPUs -> 4 v-heads, 2 qk-heads each
    for r in range(8):
        s = head_shard(32, 16, 8, r)
        assert (s.v1 - s.v0, s.q1 - s.q0) == (4, 2)
        assert s.q0 == s.v0 // 2
    with pytest.raises(ValueError):
        head_shard(32, 16, 32, 0)  # 1 v-head per rank would split a qk group
