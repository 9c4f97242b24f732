"""KV-head sharding across ranks (sharded.py), on CPU with the gloo backend:
partition, all-gather assembly in head order, stage-1 selection on every rank
and stage-2 O assembly, each compared with the unsharded oracle; and failure
detection -- a rank that leaves before a collective makes the others' next
collective end with an error under a short process-group timeout.  The
per-rank compute here is the oracle (test infrastructure), standing in for
the CUDA library."""
import datetime
import os
import socket
import traceback

import numpy as np
import pytest
import torch.multiprocessing as mp

import cases
import oracle as O
import sharded


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank, world, port, timeout_s=60):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=timeout_s))


def _run(fn, world, *args):
    """Runs fn(rank, world, port, queue, *args) on `world` spawned ranks and
    returns their queue items by rank."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=fn, args=(r, world, port, q) + args) for r in range(world)]
    for p in procs:
        p.start()
    out = {}
    for _ in range(world):
        r, item = q.get(timeout=180)
        out[r] = item
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    return out


def _both_rank(rank, world, port, q, s1_name, s2_name):
    try:
        import torch
        import torch.distributed as dist
        _init(rank, world, port)
        # stage 1
        p = dict(cases.STAGE1)[s1_name]
        Qf, Kf, _ = cases.stage1_build(p)
        cfg = cases.stage1_config(p)

        def pool_heads(h0, nh):
            rows = O.evict_pool_heads(Qf, Kf, p["len_q"], p["len_k"], cfg, h0, nh) if nh else \
                np.zeros((0, p["len_k"] - min(p["window"], p["len_q"])), np.float32)
            return torch.from_numpy(np.ascontiguousarray(rows))[None]

        def select(pooled):
            return O.evict_select_pooled(pooled[0].numpy(), p["len_q"], p["len_k"], cfg)

        kept = sharded.sharded_evict(pool_heads, select, p["HK"])
        # stage 2
        p2 = dict(cases.STAGE2)[s2_name]
        qf, Kf2, Vf = cases.stage2_build(p2)
        cfg2 = cases.stage2_config(p2)
        G = p2["H"] // p2["HK"]

        def decode_heads(h0, nh):
            # the rank sees only its shard: query heads h0*G.., KV heads h0..
            lc = O.Config(**{**cfg2.__dict__, "num_heads": nh * G, "num_heads_kv": nh})
            Ol, _ = O.hsa_decode(qf[h0 * G:(h0 + nh) * G], Kf2[h0:h0 + nh], Vf[h0:h0 + nh], p2["L"], lc,
                                 kv_bytes=2 if p2["bf16"] else 4)
            return torch.from_numpy(np.ascontiguousarray(Ol))[None]

        Og = sharded.sharded_decode(decode_heads, p2["HK"], G)
        dist.destroy_process_group()
        q.put((rank, (kept, Og[0].numpy())))
    except Exception:
        q.put((rank, traceback.format_exc()))


def _leaving_rank(rank, world, port, q):
    """Rank 1 leaves between steps without joining the collective; rank 0's
    next all-gather must end with an error, not hang."""
    try:
        import torch
        import torch.distributed as dist
        _init(rank, world, port, timeout_s=5)
        x = torch.full((1, 1, 4), float(rank))
        sharded.gather_rows(x, [1, 1])  # step 1: both ranks take part
        if rank == 1:
            q.put((rank, "left"))
            q.close()
            q.join_thread()  # the message is out before the process ends
            os._exit(0)
        try:
            sharded.gather_rows(x, [1, 1])
            q.put((rank, "no error"))
        except Exception as e:  # gloo reports the closed peer or the timeout
            q.put((rank, "error: " + type(e).__name__))
    except Exception:
        q.put((rank, traceback.format_exc()))


def test_head_range_partitions():
    for hk in range(1, 17):
        for world in range(1, 9):
            ranges = [sharded.head_range(hk, world, r) for r in range(world)]
            nxt = 0
            for h0, nh in ranges:
                assert h0 == nxt and nh >= 0
                nxt += nh
            assert nxt == hk
            assert max(n for _, n in ranges) - min(n for _, n in ranges) <= 1
    with pytest.raises(ValueError):
        sharded.head_range(8, 2, 2)


@pytest.mark.parametrize("world", [2, 3])
def test_sharded_stages_match_unsharded(world):
    s1, s2 = "s1_shortq", "s2_mha_d64"
    out = _run(_both_rank, world, s1, s2)
    p = dict(cases.STAGE1)[s1]
    Qf, Kf, _ = cases.stage1_build(p)
    want_kept = O.prefill_eviction(Qf, Kf, p["len_q"], p["len_k"], cases.stage1_config(p))
    p2 = dict(cases.STAGE2)[s2]
    qf, Kf2, Vf = cases.stage2_build(p2)
    want_o, _ = O.hsa_decode(qf, Kf2, Vf, p2["L"], cases.stage2_config(p2), kv_bytes=2 if p2["bf16"] else 4)
    for r in range(world):
        assert not isinstance(out[r], str), out[r]
        kept, o = out[r]
        np.testing.assert_array_equal(kept, want_kept)  # the same selection on every rank
        np.testing.assert_array_equal(o, want_o)  # heads are independent: identical bits


def test_rank_leaving_ends_peer_collective_with_error():
    out = _run(_leaving_rank, 2)
    assert out[1] == "left"
    assert out[0].startswith("error"), out[0]
