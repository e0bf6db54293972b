"""World-size-2 gloo run of the context-parallel orchestration on CPU.  The
CUDA compute is replaced by numpy stand-ins of the same contracts (GDN head
shard -> its outputs; GQA key shard -> (o, m, l) partials; merge of the
gathered partials); the plan and the collective sequence are the ones the GPU
path uses."""
import os
import socket

import numpy as np
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from q35attn.parallel import ShardPlan, decode_step, split_range

LOG2E = 1.4426950408889634


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _partial(q, K, V):
    """q [Hq, D], K/V [Hq, L, D] (groups expanded) -> [Hq, D+2] = o | m | l (log2 units)."""
    s = np.einsum("hd,hld->hl", q, K) * LOG2E
    m = s.max(axis=1) if s.shape[1] else np.full(q.shape[0], -np.inf)
    p = np.exp2(s - m[:, None]) if s.shape[1] else np.zeros((q.shape[0], 0))
    o = np.einsum("hl,hld->hd", p, V)
    return np.concatenate([o, m[:, None], p.sum(axis=1)[:, None]], axis=1)


def _combine(parts):
    parts = np.stack(parts)
    M = parts[:, :, -2].max(axis=0)
    w = np.exp2(parts[:, :, -2] - M)
    return (w[:, :, None] * parts[:, :, :-2]).sum(0) / (w * parts[:, :, -1]).sum(0)[:, None]


def _worker(rank, world, port, seed, q_out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    rng = np.random.RandomState(seed)
    Hq, D, L = 4, 16, 37
    q = rng.randn(Hq, D)
    K = rng.randn(Hq, L, D)
    V = rng.randn(Hq, L, D)
    gdn_full = rng.randn(16 * 8)
    plan = ShardPlan(world, rank, 16, 16, L)
    lo, hi = plan.kv_tokens
    v0, v1 = plan.gdn_v_heads

    def gather(x):
        t = torch.from_numpy(np.ascontiguousarray(x))
        out = [torch.empty_like(t) for _ in range(world)]
        dist.all_gather(out, t)
        return [o.numpy() for o in out]

    g_all, gqa = decode_step(plan, lambda: gdn_full[v0 * 8:v1 * 8], lambda: _partial(q / 4, K[:, lo:hi],
                                                                                        V[:, lo:hi]),
                             gather, _combine)
    q_out.put((rank, np.concatenate(g_all), gqa))
    dist.barrier()
    dist.destroy_process_group()


def test_context_parallel_orchestration_gloo_world2():
    world, seed = 2, 5
    ctx = mp.get_context("spawn")
    q_out = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, seed, q_out)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q_out.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    rng = np.random.RandomState(seed)
    Hq, D, L = 4, 16, 37
    q = rng.randn(Hq, D)
    K = rng.randn(Hq, L, D)
    V = rng.randn(Hq, L, D)
    gdn_full = rng.randn(16 * 8)
    s = np.einsum("hd,hld->hl", q / 4, K)
    p = np.exp(s - s.max(1, keepdims=True))
    ref = np.einsum("hl,hld->hd", p / p.sum(1, keepdims=True), V)
    for _, g_all, gqa in res:
        np.testing.assert_allclose(g_all, gdn_full)
        np.testing.assert_allclose(gqa, ref, rtol=1e-10, atol=1e-12)


def test_split_range_covers_everything():
    for n in (0, 1, 7, 32768, 32771):
        for w in (1, 2, 3, 8):
            parts = [split_range(n, w, r) for r in range(w)]
            assert parts[0][0] == 0 and parts[-1][1] == n
            assert all(parts[i][1] == parts[i + 1][0] for i in range(w - 1))
