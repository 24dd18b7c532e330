"""Expert parallelism on GPUs: pw_ep_* over NCCL, one process per GPU.

The two-GPU layer must equal pw_moe_layer on one GPU bit for bit (same
kernels, same combine order) and the oracle within the layer tolerance.
Failure handling is exercised on the host only: a peer that never joins, and
a peer that leaves between layers; no GPU is faulted (NVLS off).
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

E, HID, INTER = 16, 1024, 512


def _bank(dev, experts):
    from mimo_prismwing_b200 import synth
    return [synth.expert(HID, INTER, 900 + e, dev) for e in experts]


def _worker(rank, world, uid_q, res_q, tokens_per_rank, mode, nccl=False):
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    try:
        torch.cuda.set_device(rank)
        dev = f"cuda:{rank}"
        from mimo_prismwing_b200 import synth
        from mimo_prismwing_b200.runtime import WideMoeRuntime
        rt = WideMoeRuntime.compile_with_fused_gate_up(rank)
        if rank == 0:
            uid = WideMoeRuntime.ep_unique_id()
            for _ in range(world - 1):
                uid_q.put(uid)
        else:
            uid = uid_q.get(timeout=60)
        rt.ep_init(rank, world, uid, timeout_ms=8000 if mode == "leave" else 20000, max_tokens=512,
                   hidden=HID, local_experts=E // world, nccl_transport=nccl)
        L = E // world
        local = rt.create_bank(_bank(dev, range(rank * L, (rank + 1) * L)))
        w, bias = synth.router(E, HID, 77, dev)
        T = tokens_per_rank[rank]
        x = synth.activations(max(T, 1), HID, 300 + rank, dev)[:T]
        if mode == "leave":
            def report_and_exit(val):
                res_q.put((rank, val))
                res_q.close()
                res_q.join_thread()  # flush the queue's feeder thread before _exit
                os._exit(0)
            if rank == 1:
                torch.cuda.synchronize()
                report_and_exit("left")  # between steps: nothing in flight
            import time
            time.sleep(2.0)
            try:
                rt.ep_moe_layer(x, w, bias, local)
                report_and_exit("no error")
            except Exception as exc:  # expected: bounded timeout / NCCL error
                report_and_exit(getattr(exc, "status", str(exc)))
        ex = rt.ep_moe_layer(x, w, bias, local, want_routes=True)
        # the asynchronous form (enqueue and return) gives the same bits; a
        # synchronous call after it observes its completion
        y_async = torch.empty((T, HID), device=dev)
        rt.ep_moe_layer(x, w, bias, local, asynchronous=True, out=y_async)
        rt.ep_moe_layer(x, w, bias, local)
        # the decoder-layer block (RMSNorm before, residual add after) on the
        # same ranks: collective too
        nw = (1.0 + 0.1 * torch.randn(HID, generator=torch.Generator().manual_seed(5))).to(torch.bfloat16).cuda(rank)
        blk = rt.moe_block(x, nw, 1e-5, w, bias, local, expert_parallel=True)
        if T == 0:
            res_q.put((rank, "ok"))
            return
        assert torch.equal(y_async, ex.output), "asynchronous EP layer differs"
        y = ex.output.cpu().numpy()
        sel = ex.selected.cpu().numpy().astype(np.uint32)
        wts = ex.weights.cpu().numpy()
        # the same tokens through the single-GPU layer with all experts ...
        import sys
        sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
        from gpu_helpers import assert_close_bf16, bank_arrays
        from oracle import oracle as O
        full_bank = _bank(dev, range(E))
        rt1 = WideMoeRuntime.compile_with_fused_gate_up(rank)
        full_handle = rt1.create_bank(full_bank)
        single = rt1.moe_layer(x, w, bias, full_handle).output.cpu().numpy()
        single_blk = rt1.moe_block(x, nw, 1e-5, w, bias, full_handle).output.cpu().numpy()
        # bit-identical when both pick the same expert kernels: the single-GPU
        # layer runs the tcgen05 GEMM from 256 tokens, the expert-parallel one
        # when an expert receives > 16 rows (GEMV and GEMM sum in different orders)
        total = sum(tokens_per_rank)
        if T >= 256 or total * 8 <= 16 * E // 4:
            assert np.array_equal(y.view(np.uint32), single.view(np.uint32)), "EP != single GPU"
            assert np.array_equal(blk.output.cpu().numpy().view(np.uint32), single_blk.view(np.uint32)), \
                "EP block != single-GPU block"
        # ... and the oracle
        ref = O.routed_layer(x.cpu().numpy(), sel, wts, bank_arrays(full_bank), O.ACC_F64, O.EXP_SLEEF)
        assert_close_bf16(y, ref, what=f"EP layer rank {rank}")
        res_q.put((rank, "ok"))
    except BaseException as exc:
        res_q.put((rank, f"error: {exc!r}"))
        raise


def _run(world, tokens_per_rank, mode, wait_s=300, nccl=False):
    ctx = mp.get_context("spawn")
    uid_q, res_q = ctx.Queue(), ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, uid_q, res_q, tokens_per_rank, mode, nccl))
             for r in range(world)]
    for p in procs:
        p.start()
    out = {}
    for _ in range(world):
        rank, val = res_q.get(timeout=wait_s)
        out[rank] = val
    for p in procs:
        p.join(timeout=120)
        if p.is_alive():
            p.kill()
    return out


def test_ep_init_times_out_without_peer():
    # rank 0 of 2 joins alone: the bounded, non-blocking init gives up
    from mimo_prismwing_b200.runtime import PrismwingError, WideMoeRuntime
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    rt = WideMoeRuntime.compile(0)
    uid = WideMoeRuntime.ep_unique_id()
    with pytest.raises(PrismwingError) as err:
        rt.ep_init(0, 2, uid, timeout_ms=3000)
    assert err.value.status == -7
    rt.close()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("transport", ["p2p", "nccl"])
@pytest.mark.parametrize("tokens_per_rank", [(4, 4), (3, 0), (300, 200)])
def test_ep_layer_two_gpus(tokens_per_rank, transport):
    out = _run(2, tokens_per_rank, "layer", nccl=transport == "nccl")
    assert out == {0: "ok", 1: "ok"}, out


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_ep_peer_leaves_between_layers():
    # the survivor's layer must end within its 8 s deadline (plus start-up)
    out = _run(2, (4, 4), "leave", wait_s=90)
    assert out[1] == "left"
    assert out[0] in (-7, -6), out[0]  # PW_ERR_TIMEOUT or PW_ERR_NCCL, within the deadline
