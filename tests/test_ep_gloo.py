"""Expert-parallel dispatch / combine on CPU (the torch-only stand-in of
tests/ep_cpu_exchange.py): gloo ranks, the numpy oracle
as each rank's local forward, checked against one single-process oracle
forward of all tokens.  Per expert the INT8 activations, mm1 and a2q rows
are bit-identical; the combined output is within the reference tolerance
(only the cross-rank summation order differs)."""

import os
import socket
import traceback

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

WORLD = 2


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _np(t):
    return t.float().numpy() if t.is_floating_point() else t.numpy()


def _worker(rank, world, port, cfg_name, only_rank0_experts, errq):
    try:
        import datetime
        import torch.distributed as dist
        from oracle import ref_cpu as ref
        from tests.helpers import load_workloads
        from tests.ep_cpu_exchange import CPUExchange

        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        dist.init_process_group("gloo", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=60))
        wl = load_workloads()
        cfg = wl.CONFIGS[cfg_name]
        inp = wl.make_inputs(cfg)
        ids = inp["topk_ids"]
        if only_rank0_experts:  # every token on rank 0's experts: rank 1 receives nothing
            ids = ids % (cfg.E // world)
        T, k = ids.shape
        tm = ref.VARIANT_TILE_M[ref.pick_grouped_hybrid_variant(T * k, cfg.E)]
        ep = CPUExchange(cfg.E)
        lo, n = ep.first, ep.n_local
        per = T // world
        sl = slice(rank * per, (rank + 1) * per)
        emap = ep.expert_map("cpu").numpy()
        npw = {kk: _np(v) for kk, v in inp.items()}
        traces = {}

        def local_forward(h, i, w):
            if h.shape[0] == 0:
                return torch.empty(0, h.shape[1], dtype=h.dtype)
            tr = ref.moe_forward(
                _np(h), npw["w13"][lo:lo + n], npw["w2"][lo:lo + n], _np(i), _np(w),
                npw["w13_q"][lo:lo + n], npw["w13_f"][lo:lo + n], npw["w2_q"][lo:lo + n],
                npw["w2_f"][lo:lo + n], dtype=cfg.dtype, global_num_experts=cfg.E,
                expert_map=emap, super_group_size=cfg.sg, q_max=cfg.q_max, trace=True,
                tile_m=tm)
            traces["t"] = tr
            return torch.from_numpy(tr.out).to(h.dtype)

        out = ep.forward(inp["hidden"][sl], ids[sl], inp["topk_weights"][sl], local_forward)
        gathered = [torch.empty_like(out) for _ in range(world)]
        dist.all_gather(gathered, out)
        full = ref.moe_forward(npw["hidden"], npw["w13"], npw["w2"], _np(ids),
                               npw["topk_weights"], npw["w13_q"], npw["w13_f"], npw["w2_q"],
                               npw["w2_f"], dtype=cfg.dtype, global_num_experts=cfg.E,
                               super_group_size=cfg.sg, q_max=cfg.q_max, trace=True)
        got = torch.cat(gathered).float().numpy()
        rel = np.abs(got - full.out).max() / np.abs(full.out).max()
        assert rel <= 1e-2, f"rank {rank}: EP output max-abs-rel {rel:.3e} > 1e-2"
        if "t" in traces:
            loc = traces["t"]
            for le in range(n):
                e = lo + le
                a, b = int(loc.offsets[le]), int(loc.offsets[le + 1])
                fa, fb = int(full.offsets[e]), int(full.offsets[e + 1])
                assert b - a == fb - fa, f"expert {e}: {b - a} rows vs {fb - fa}"
                for name in ("a1q", "mm1", "a2q", "mm2"):
                    np.testing.assert_array_equal(getattr(loc, name)[a:b],
                                                  getattr(full, name)[fa:fb],
                                                  err_msg=f"{name} of expert {e}")
        else:
            assert int(full.offsets[lo + n] - full.offsets[lo]) == 0
        dist.destroy_process_group()
    except BaseException:
        errq.put(f"rank {rank}:\n{traceback.format_exc()}")
        raise


@pytest.mark.parametrize("world,cfg_name,only_rank0", [(WORLD, "tiny", False),
                                                        (WORLD, "mid", False),
                                                        (WORLD, "tiny", True),
                                                        (4, "tiny", False), (4, "mid", False)])
def test_ep_gloo_ranks_match_single_process(world, cfg_name, only_rank0):
    """world gloo ranks on CPU: the exchange orders every expert's rows as one
    process would (bit-identical activations, accumulators and outputs per
    expert), the combined output is within 1e-2 of the single-process one."""
    ctx = mp.get_context("spawn")
    errq = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, cfg_name, only_rank0, errq))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
    errs = []
    while not errq.empty():
        errs.append(errq.get())
    assert not alive, "EP ranks did not finish"
    assert not errs, "\n".join(errs)
    assert all(p.exitcode == 0 for p in procs)
