"""Expert parallelism on two GPUs, over NCCL and over NVLink peer memory.
Each rank runs the EP forward (dispatch -> sm_100a forward of its local
experts -> combine) and, on its own GPU, the single-GPU forward of all
tokens; per local expert the INT8 activations, mm1, a2q and mm2 rows must be
bit-identical.  The combined output must equal the single-GPU output bit for
bit with the peer exchange's top-k combine (the unpermute runs whole on the
token's own rank), and agree within the reference tolerance (max-abs-rel
1e-2) with the partial-row combines (NCCL, and the peer exchange's "rows"
mode), which add per-rank partial sums.  The peer-memory exchange also runs
steps of both parities and two steps captured in a CUDA graph and replayed.
The two-rank tests need two GPUs and are skipped otherwise; the one-GPU
tests below drive the peer kernels over two local regions."""

import os
import socket
import traceback

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu
WORLD = 2


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, cfg_name, mode, errq):
    try:
        import datetime
        from dataclasses import replace
        import torch.distributed as dist
        import int8blockwisegemm_b200 as pkg
        from int8blockwisegemm_b200.ep import EPMoE, ExpertParallel, global_tile_m
        from tests.helpers import load_workloads

        os.environ["MASTER_ADDR"] = "127.0.0.1"
        os.environ["MASTER_PORT"] = str(port)
        torch.cuda.set_device(rank)
        dev = torch.device("cuda", rank)
        dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                                timeout=datetime.timedelta(seconds=120))
        wl = load_workloads()
        cfg = wl.CONFIGS[cfg_name]
        inp = wl.make_inputs(cfg)
        r = pkg.cutlass_runner
        r._USE_FUSED_PERMUTE_QUANT_W1 = True
        r._USE_FUSED_SILU_QUANT_W2 = True
        T, k = inp["topk_ids"].shape
        d = {kk: v.to(dev) for kk, v in inp.items()}
        dt = d["hidden"].dtype
        # single-GPU reference forward of all tokens, on this rank's GPU
        full_tr = {}
        full_out = torch.empty(T, cfg.K, dtype=dt, device=dev)
        r._run_cutlass_int8_hybrid_grouped_moe(
            full_out, d["hidden"], d["w13"], d["w2"], d["topk_ids"], d["topk_weights"],
            pkg.activation.MoEActivation.SILU, cfg.E, None, d["w13_q"], d["w13_f"], d["w2_q"],
            d["w2_f"], torch.empty(T * k, max(2 * cfg.N, cfg.K), dtype=dt, device=dev),
            torch.empty(T * k, max(cfg.N, cfg.K), dtype=dt, device=dev), cfg.quant_block,
            cfg.sg, cfg.q_max, _trace=full_tr)
        ep = ExpertParallel(cfg.E)
        moe = EPMoE(ep, d["w13"], d["w2"], d["w13_q"], d["w13_f"], d["w2_q"], d["w2_f"],
                    quant_block_size=cfg.quant_block, super_group_size=cfg.sg,
                    q_max=cfg.q_max, tile_m=global_tile_m(T, k, cfg.E))
        per = T // world
        sl = slice(rank * per, (rank + 1) * per)
        h_in = d["hidden"][sl].contiguous()
        i_in = d["topk_ids"][sl].contiguous()
        w_in = d["topk_weights"][sl].contiguous()
        p2p = mode.startswith("p2p")
        if p2p:
            moe.enable_peer_exchange(per, cfg.K, k, dt,
                                     combine="rows" if mode == "p2p_rows" else "topk")
            assert moe.p2p.combine == ("rows" if mode == "p2p_rows" else "topk")
        tr = {}
        out = moe.forward(h_in, i_in, w_in, trace=tr)
        torch.cuda.synchronize()
        ref = full_out[sl].float()

        def check(o, what):
            if mode == "p2p":  # top-k combine: the single-GPU arithmetic
                assert torch.equal(o, full_out[sl]), f"rank {rank} {what}: EP output differs"
                return
            rel = ((o.float() - ref).abs().max() / ref.abs().max()).item()
            assert rel <= 1e-2, f"rank {rank} {what}: EP output max-abs-rel {rel:.3e} > 1e-2"

        check(out, "first step")
        assert tr["tile_m"] == full_tr["tile_m"]
        leo, feo = tr["eft"].cpu(), full_tr["eft"].cpu()
        for le in range(ep.n_local):
            e = ep.first + le
            a, b = int(leo[le]), int(leo[le + 1])
            fa, fb = int(feo[e]), int(feo[e + 1])
            assert b - a == fb - fa, f"expert {e}: {b - a} rows vs {fb - fa}"
            for name in ("a1q", "mm1", "a2q", "mm2"):
                if tr[name] is None:  # mm1 is not materialised by the fused w13 epilogue
                    assert full_tr[name] is None
                    continue
                assert torch.equal(tr[name][a:b], full_tr[name][fa:fb]), f"{name} of expert {e}"
        if p2p:
            # the other step parity, eagerly; then two steps in a CUDA graph
            first = out.clone()
            out2 = moe.forward(h_in, i_in, w_in)
            torch.cuda.synchronize()
            assert torch.equal(out2, first), "second step differs"
            o_g = torch.empty_like(first)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                moe.forward(h_in, i_in, w_in, out=o_g)
                moe.forward(h_in, i_in, w_in, out=o_g)
            for _ in range(3):
                o_g.zero_()
                dist.barrier()
                g.replay()
                torch.cuda.synchronize()
                assert torch.equal(o_g, first), "graph replay differs"
            del g
            moe.p2p.close()
        assert pkg._lib.device_error(rank) == 0
        dist.barrier()
        dist.destroy_process_group()
    except BaseException:
        errq.put(f"rank {rank}:\n{traceback.format_exc()}")
        raise


@pytest.mark.parametrize("mode", ["nccl", "p2p", "p2p_rows"])
@pytest.mark.parametrize("cfg_name", ["mid", "default"])
def test_ep_two_gpus_matches_single_gpu(cfg_name, mode):
    if torch.cuda.device_count() < WORLD:
        pytest.skip(f"needs {WORLD} GPUs")
    ctx = mp.get_context("spawn")
    errq = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, WORLD, port, cfg_name, mode, errq))
             for r in range(WORLD)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=600)
    alive = [p for p in procs if p.is_alive()]
    for p in alive:
        p.kill()
    errs = []
    while not errq.empty():
        errs.append(errq.get())
    assert not alive, "EP ranks did not finish"
    assert not errs, "\n".join(errs)
    assert all(p.exitcode == 0 for p in procs)


def test_p2p_dispatch_peer_timeout_one_gpu():
    """A peer that never answers, on one GPU: rank 1's region is a second
    local region that nothing writes, so rank 0's dispatch waits for segment
    lengths that never come.  Every wait gives up after its bound (2 s), the
    kernel returns, the device error word reports the peer timeout, and the
    persistent CTA completion counter is back at zero after each such step
    (every CTA counts itself even when its wait failed), so a later step
    cannot raise its "rows posted" flag early."""
    import ctypes

    import int8blockwisegemm_b200 as pkg
    from int8blockwisegemm_b200._lib import call
    from int8blockwisegemm_b200.ep import _Layout, _P2PDesc

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    P, T, k, K = 2, 64, 4, 256
    lay = _Layout()
    call("i8moe_ep_p2p_region_bytes", P, P * T, k, K, 2, 0, ctypes.addressof(lay))
    regions = [torch.zeros(lay.bytes, dtype=torch.uint8, device=dev) for _ in range(P)]
    desc = _P2PDesc()
    for d in range(P):
        desc.bases[d] = regions[d].data_ptr()
    desc.n_rank, desc.rank, desc.n_token, desc.capacity = P, 0, T, P * T
    desc.topk, desc.n_hidden, desc.elem_bytes, desc.pad_expert = k, K, 2, 8
    desc.layout = lay
    g = torch.Generator().manual_seed(0)
    ids = torch.randint(0, 16, (T, k), generator=g, dtype=torch.int32).to(dev)
    w = torch.rand(T, k, generator=g).to(dev)
    hidden = torch.randn(T, K, generator=g).to(torch.bfloat16).to(dev)
    pos = torch.empty(T, P, dtype=torch.int32, device=dev)
    lst = torch.empty(P, T, dtype=torch.int32, device=dev)
    counts = torch.empty(P, dtype=torch.int32, device=dev)
    st = torch.cuda.current_stream(dev).cuda_stream
    pkg._lib.device_error(0, clear=True)
    ctr_off = lay.off_epoch + 8
    for step in range(2):
        call("i8moe_ep_plan", ids.data_ptr(), T, k, 8, P, pos.data_ptr(), lst.data_ptr(),
             counts.data_ptr(), st)
        call("i8moe_ep_p2p_dispatch", ctypes.addressof(desc), step & 1, hidden.data_ptr(),
             ids.data_ptr(), w.data_ptr(), lst.data_ptr(), counts.data_ptr(), st)
        torch.cuda.synchronize()
        err = pkg._lib.device_error(0, clear=True)
        assert err & (1 << 6), f"step {step}: no peer-timeout bit in the error word ({err:#x})"
        ctr = regions[0][ctr_off:ctr_off + 4].view(torch.int32).item()
        assert ctr == 0, f"step {step}: CTA completion counter left at {ctr}"
        epoch = regions[0][lay.off_epoch:lay.off_epoch + 8].view(torch.int64).item()
        assert epoch == step + 1
    assert pkg._lib.device_error(0) == 0


def test_p2p_combine_topk_one_gpu():
    """The top-k combine kernel over two local regions, as rank 1 of 2.
    Both destinations' mm2 rows and inverse maps are filled on the host, the
    segment lengths rank 0 sent to each destination go into rank 1's inbox
    (so rank 1's segments start past them), and every "output ready" flag is
    raised before the launch, so no wait spins.  The output must equal the
    single-GPU unpermute of the same rows (the same fma chain in top-k
    order), for both step parities."""
    import ctypes

    import int8blockwisegemm_b200 as pkg
    from int8blockwisegemm_b200._lib import BF16, call
    from int8blockwisegemm_b200.ep import COMBINE_TOPK, _Layout, _P2PDesc
    from int8blockwisegemm_b200.permute import moe_unpermute

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    P, T, k, K, E = 2, 64, 4, 256, 16
    n_local, C = E // P, P * T
    lay = _Layout()
    call("i8moe_ep_p2p_region_bytes", P, C, k, K, 2, COMBINE_TOPK, ctypes.addressof(lay))
    assert lay.out_bytes == 0 and lay.mm2_bytes >= C * k * K * 2 and lay.inv_bytes >= C * k * 4
    regions = [torch.zeros(lay.bytes, dtype=torch.uint8, device=dev) for _ in range(P)]
    desc = _P2PDesc()
    for d in range(P):
        desc.bases[d] = regions[d].data_ptr()
    desc.n_rank, desc.rank, desc.n_token, desc.capacity = P, 1, T, C
    desc.topk, desc.n_hidden, desc.elem_bytes, desc.pad_expert = k, K, 2, 0
    desc.layout = lay
    g = torch.Generator().manual_seed(3)
    # distinct experts per token, as top-k gives
    ids = torch.stack([torch.randperm(E, generator=g)[:k] for _ in range(T)]).to(torch.int32)
    w = torch.rand(T, k, generator=g)
    owner = ids // n_local
    pos = torch.full((T, P), -1, dtype=torch.int32)  # slot in each destination's segment
    for dd in range(P):
        members = (owner == dd).any(dim=1).nonzero().flatten()
        pos[members, dd] = torch.arange(members.numel(), dtype=torch.int32)
    sent_by_rank0 = [5, 9]  # rows rank 0 placed first in each destination's receive buffer
    st = torch.cuda.current_stream(dev).cuda_stream
    pkg._lib.device_error(0, clear=True)
    for step in range(2):
        par = step & 1
        mm2 = [torch.randn(C * k, K, generator=g).to(torch.bfloat16) for _ in range(P)]
        gathered = torch.empty(T * k, K, dtype=torch.bfloat16)
        for dd in range(P):
            inv = torch.full((C * k,), -1, dtype=torch.int32)
            perm = torch.randperm(C * k, generator=g).to(torch.int32)
            inv[:] = perm  # any row of mm2; every slot reads one
            r = regions[dd]
            r[lay.off_mm2 + par * lay.mm2_bytes:][:C * k * K * 2].copy_(
                mm2[dd].view(torch.uint8).flatten().to(dev))
            r[lay.off_inv + par * lay.inv_bytes:][:C * k * 4].copy_(
                inv.view(torch.uint8).to(dev))
            for t in range(T):
                for j in range(k):
                    if owner[t, j] == dd:
                        row = sent_by_rank0[dd] + int(pos[t, dd])
                        gathered[t * k + j] = mm2[dd][int(inv[row * k + j])]
        inbox = torch.zeros(2, P, P, dtype=torch.int32)
        inbox[par, 0] = torch.tensor(sent_by_rank0, dtype=torch.int32)
        r1 = regions[1]
        r1[lay.off_inbox:][:2 * P * P * 4].copy_(inbox.view(torch.uint8).flatten().to(dev))
        flags = torch.full((3, P), step + 1, dtype=torch.int64)
        r1[lay.off_flags:][:3 * P * 8].copy_(flags.view(torch.uint8).flatten().to(dev))
        r1[lay.off_epoch:][:8].copy_(torch.tensor([step + 1], dtype=torch.int64)
                                     .view(torch.uint8).to(dev))
        ids_d, w_d, pos_d = ids.to(dev), w.to(dev), pos.to(dev)
        out = torch.empty(T, K, dtype=torch.bfloat16, device=dev)
        call("i8moe_ep_p2p_combine_topk", ctypes.addressof(desc), par, BF16, pos_d.data_ptr(),
             ids_d.data_ptr(), w_d.data_ptr(), n_local, out.data_ptr(), st)
        ref = torch.empty(T, K, dtype=torch.bfloat16, device=dev)
        moe_unpermute(ref, gathered.to(dev), w_d, torch.arange(T * k, dtype=torch.int32,
                                                                 device=dev))
        torch.cuda.synchronize()
        assert pkg._lib.device_error(0, clear=True) == 0
        assert torch.equal(out, ref), f"step {step}: top-k combine differs from the unpermute"
