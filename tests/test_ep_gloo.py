"""Expert parallelism, host side, on CPU: two gloo ranks run the data flow of
pw_ep_moe_layer with the real transfer planner (pw_ep_plan from the C ABI)
and the oracle for the expert arithmetic, and each rank's output must equal
the single-process oracle routed layer on its tokens bit for bit.

What this pins: the expert partition (rank g owns [g L, (g+1) L)), the
all-gathered offsets -> send/recv sizes, the permutation into expert order,
the scatter back into received order and the source-side combine in
ascending expert order.  The CUDA kernels are covered by the GPU tests.
"""
import ctypes
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

E, HID, INTER = 16, 512, 256


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _bank():
    from mimo_prismwing_b200 import synth
    out = []
    for e in range(E):
        g, u, d = synth.expert(HID, INTER, 900 + e, "cpu")
        out.append(tuple(t.numpy() for p in (g, u, d) for t in (p.weight, p.scale)))
    return out


def _plan(all_off, world, rank):
    from mimo_prismwing_b200 import _lib
    L = _lib.load()
    all_off = np.ascontiguousarray(all_off, dtype=np.uint32)
    Lx = E // world
    rows = int(sum(all_off[g, (rank + 1) * Lx] - all_off[g, rank * Lx] for g in range(world)))
    n_send = np.zeros(world, np.uint32)
    n_recv = np.zeros(world, np.uint32)
    base = np.zeros(world + 1, np.uint32)
    perm = np.zeros(max(rows, 1), np.uint32)
    eb = np.zeros(Lx + 1, np.uint32)
    p = lambda a: a.ctypes.data_as(ctypes.c_void_p)
    rc = L.pw_ep_plan(p(all_off), world, rank, E, p(n_send), p(n_recv), p(base), p(perm), p(eb))
    assert rc == 0
    return n_send, n_recv, base, perm[:rows], eb


def _expert_rows(bank_e, codes, scales):
    from oracle import oracle as O
    gw, gs, uw, us, dw, ds = bank_e
    gate = O.blockscaled_linear(gw, gs, codes, scales, mode=O.ACC_F64)
    up = O.blockscaled_linear(uw, us, codes, scales, mode=O.ACC_F64)
    act = O.staged_swiglu(gate, up, O.EXP_SLEEF)
    hc, hs, _ = O.dynamic_fp8(act)
    return O.round_bf16(O.blockscaled_linear(dw, ds, hc, hs, mode=O.ACC_F64))


def _rank_main(rank, world, port, tokens_per_rank, errq):
    try:
        os.environ.setdefault("OMP_NUM_THREADS", "2")
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
        from mimo_prismwing_b200 import synth
        from oracle import oracle as O
        bank = _bank()
        w, bias = synth.router(E, HID, 77, "cpu")
        wbits = w.view(torch.int16).numpy().view(np.uint16)
        T = tokens_per_rank[rank]
        Lx = E // world
        x = synth.activations(max(T, 1), HID, 300 + rank, "cpu").numpy()[:T]
        # 1. route + schedule (expert-major) + codes of the placements
        if T:
            sel, wts, _, _, _ = O.noaux_topk(O.router_logits(x, wbits), bias.numpy())
            offsets, order = O.schedule(sel, E)
            xc, xs, _ = O.dynamic_fp8(x)
            send_codes = xc[order // 8]
            send_scales = xs[order // 8]
        else:
            offsets = np.zeros(E + 1, np.uint32)
            order = np.zeros(0, np.uint32)
            send_codes = np.zeros((0, HID), np.uint8)
            send_scales = np.zeros((0, HID // 128), np.float32)
        # 2. all-gather the offsets, plan
        gathered = [torch.zeros(E + 1, dtype=torch.int64) for _ in range(world)]
        dist.all_gather(gathered, torch.from_numpy(offsets.astype(np.int64)))
        all_off = np.stack([g.numpy() for g in gathered]).astype(np.uint32)
        n_send, n_recv, base, perm, eb = _plan(all_off, world, rank)
        assert int(n_send.sum()) == T * 8
        # 3. dispatch
        rc = torch.empty((int(n_recv.sum()), HID), dtype=torch.uint8)
        dist.all_to_all_single(rc, torch.from_numpy(np.ascontiguousarray(send_codes)),
                               [int(v) for v in n_recv], [int(v) for v in n_send])
        rs = torch.empty((int(n_recv.sum()), HID // 128), dtype=torch.float32)
        dist.all_to_all_single(rs, torch.from_numpy(np.ascontiguousarray(send_scales)),
                               [int(v) for v in n_recv], [int(v) for v in n_send])
        rc, rs = rc.numpy(), rs.numpy()
        # 4. local experts in expert order, scattered back to received order
        ret_send = np.zeros((len(perm), HID), np.float32)
        for le in range(Lx):
            a, b = int(eb[le]), int(eb[le + 1])
            if b > a:
                rows = perm[a:b]
                ret_send[rows] = _expert_rows(bank[rank * Lx + le], rc[rows], rs[rows])
        # 5. return
        ret = torch.empty((T * 8, HID), dtype=torch.float32)
        dist.all_to_all_single(ret, torch.from_numpy(ret_send), [int(v) for v in n_send],
                               [int(v) for v in n_recv])
        ret = ret.numpy()
        # 6. combine in ascending expert order, then bf16
        if T:
            y = np.zeros((T, HID), np.float32)
            place = np.empty(T * 8, np.int64)
            place[order] = np.arange(T * 8)
            for t in range(T):
                for k in np.argsort(sel[t], kind="stable"):
                    p = place[t * 8 + k]
                    y[t] = (y[t] + (ret[p] * np.float32(wts[t, k])).astype(np.float32)).astype(np.float32)
            y = O.round_bf16(y)
            ref = O.routed_layer(x, sel, wts, bank, O.ACC_F64, O.EXP_SLEEF)
            assert np.array_equal(y.view(np.uint32), ref.view(np.uint32)), f"rank {rank}: EP != single process"
        dist.barrier()
        dist.destroy_process_group()
    except BaseException as exc:  # report to the parent, which fails the test
        errq.put(f"rank {rank}: {exc!r}")
        raise


@pytest.mark.parametrize("tokens_per_rank", [(6, 3), (5, 0)])
def test_ep_host_flow_two_gloo_ranks(tokens_per_rank):
    ctx = mp.get_context("spawn")
    errq = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, tokens_per_rank, errq)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
    for p in procs:
        if p.is_alive():
            p.kill()
    errors = []
    while not errq.empty():
        errors.append(errq.get())
    assert not errors, errors
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]


def test_ep_plan_rejects_bad_offsets():
    from mimo_prismwing_b200 import _lib
    L = _lib.load()
    off = np.array([[0, 3, 2] + [2] * (E - 2)], dtype=np.uint32)  # decreasing: invalid
    z = np.zeros(8, np.uint32)
    p = lambda a: a.ctypes.data_as(ctypes.c_void_p)
    assert L.pw_ep_plan(p(off), 1, 0, E, p(z), p(z), p(z), p(z), p(z)) == -8
    assert L.pw_ep_plan(p(off), 0, 0, E, p(z), p(z), p(z), p(z), p(z)) == -1
