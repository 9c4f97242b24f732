"""KV-head sharding on GPUs (sharded.HeadShardedRocket over NCCL): each rank
holds only its heads' Q/K/V rows; stage-1 kept indices and stage-2 O must
equal the unsharded single-GPU results (stage 2 per head is independent, so
O is bit-identical).  One rank per visible GPU, at most two; with a single
GPU the driver runs as a world of one."""
import datetime
import os
import socket
import traceback

import numpy as np
import pytest
import torch.multiprocessing as mp

import cases
import rkvgen

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _to_rkv(cfg):
    import rocketkv_b200 as rkv
    return rkv.RocketConfig(**{f: getattr(cfg, f) for f in cfg.__dataclass_fields__})


def _rank(rank, world, port, q):
    try:
        import torch
        import torch.distributed as dist
        import rocketkv_b200 as rkv
        import sharded
        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                                device_id=dev)
        # stage 1: fp32, the s1_basic case
        p = dict(cases.STAGE1)["s1_basic"]
        Qf, Kf, _ = cases.stage1_build(p)
        cfg = _to_rkv(cases.stage1_config(p))
        G = p["H"] // p["HK"]
        sh = sharded.HeadShardedRocket(cfg, dev)
        h0, nh = sh.h0, sh.nh
        Ql = torch.from_numpy(np.ascontiguousarray(Qf[h0 * G:(h0 + nh) * G]))[None].to(dev)
        Kl = torch.from_numpy(np.ascontiguousarray(Kf[h0:h0 + nh]))[None].to(dev)
        kept, n = sh.evict(Ql, Kl, p["len_q"], p["len_k"], rkv.F32)
        kept = kept[0, : int(n[0])].cpu().numpy().copy()
        # stage 2: bf16, headline geometry on a short cache
        p2 = dict(cases.STAGE2)["s2_cfg1"]
        qf, K2, V2 = cases.stage2_build(p2)
        cfg2 = _to_rkv(cases.stage2_config(p2))
        sh2 = sharded.HeadShardedRocket(cfg2, dev)
        b = lambda a: torch.from_numpy(rkvgen.bf16_bits(np.ascontiguousarray(a))).view(torch.bfloat16)[None].to(dev)
        h0, nh = sh2.h0, sh2.nh
        O = sh2.decode(b(qf[h0 * G:(h0 + nh) * G]), b(K2[h0:h0 + nh]), b(V2[h0:h0 + nh]), p2["L"], 32)
        O = O[0].cpu().numpy().copy()
        # the unsharded results on this rank's GPU
        ev = rkv.Evictor(cfg, p["len_q"], p["len_k"], 1, rkv.F32, dev)
        k1, n1 = ev(torch.from_numpy(Qf)[None].to(dev), torch.from_numpy(Kf)[None].to(dev))
        want_kept = k1[0, : int(n1[0])].cpu().numpy()
        dec = rkv.HsaDecoder(cfg2, p2["L"], 1, dev, recent_window=32)
        want_O = dec(b(qf), b(K2), b(V2))[0].cpu().numpy()
        torch.cuda.synchronize()
        dist.destroy_process_group()
        q.put((rank, (kept, want_kept, O, want_O)))
    except Exception:
        q.put((rank, traceback.format_exc()))


def test_head_sharded_equals_unsharded(cuda):
    import torch
    world = min(2, torch.cuda.device_count())
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = {}
    for _ in range(world):
        r, item = q.get(timeout=300)
        out[r] = item
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    for r in range(world):
        assert not isinstance(out[r], str), out[r]
        kept, want_kept, O, want_O = out[r]
        np.testing.assert_array_equal(kept, want_kept)
        np.testing.assert_array_equal(O, want_O)
