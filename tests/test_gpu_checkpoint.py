"""Checkpoint ingestion on the GPU: a synthetic MiMo-style checkpoint written
with the safetensors library (the checkpoint's own format and tensor names,
src/text_endpoint.rs:3067 for the "_scale_inv" grids) is mapped, validated
and uploaded by the library (pw_bank_load, pw_tensor_upload), and the routed
layer over it must equal, bit for bit, the same layer over the same tensors
registered from torch (pw_bank_create).  PWEXPRT1 containers of the experts
load the same way.
"""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

LAYER, E, HID, INTER = 5, 16, 1024, 512


def _checkpoint(tmp_path, bad_byte=False):
    """Two shards: experts 0-7 + router in the first, experts 8-15 + norm in the second."""
    import safetensors.torch as st
    from mimo_prismwing_b200 import synth
    shards = [{}, {}]
    experts = []
    for e in range(E):
        trio = synth.expert(HID, INTER, 3000 + e, "cpu")
        experts.append(trio)
        for name, p in zip(("gate_proj", "up_proj", "down_proj"), trio):
            key = f"model.layers.{LAYER}.mlp.experts.{e}.{name}.weight"
            w = p.weight.clone()
            if bad_byte and e == 11 and name == "up_proj":
                w[3, 7] = 0x7F
            shards[e // 8][key] = w.view(torch.float8_e4m3fn)
            shards[e // 8][key + "_scale_inv"] = p.scale.clone()
    rw, rb = synth.router_f32(E, HID, 91, "cpu")
    shards[0][f"model.layers.{LAYER}.mlp.gate.weight"] = rw
    shards[0][f"model.layers.{LAYER}.mlp.gate.e_score_correction_bias"] = rb
    nw = (1.0 + 0.1 * torch.randn(HID)).to(torch.bfloat16)
    shards[1][f"model.layers.{LAYER}.post_attention_layernorm.weight"] = nw
    paths = []
    for i, sh in enumerate(shards):
        p = str(tmp_path / f"model-0000{i + 1}-of-00002.safetensors")
        st.save_file(sh, p)
        paths.append(p)
    return paths, experts, (rw, rb, nw)


@pytest.fixture(scope="module")
def rt():
    from mimo_prismwing_b200.runtime import WideMoeRuntime
    r = WideMoeRuntime.compile_with_fused_gate_up(0)
    yield r
    r.close()


def test_bank_from_safetensors_equals_bank_from_torch(rt, tmp_path):
    from mimo_prismwing_b200 import checkpoint as C
    from mimo_prismwing_b200 import synth
    paths, experts, (rw, rb, nw) = _checkpoint(tmp_path)
    files = [C.MappedSafetensors.open(p) for p in paths]
    bank = C.load_bank(rt, files, LAYER, 0, E)
    wbuf = C.upload(rt, files, f"model.layers.{LAYER}.mlp.gate.weight", "F32", (E, HID))
    bbuf = C.upload(rt, files, f"model.layers.{LAYER}.mlp.gate.e_score_correction_bias", "F32", (E,))
    nbuf = C.upload(rt, files, f"model.layers.{LAYER}.post_attention_layernorm.weight", "BF16", (HID,))
    w = torch.as_tensor(wbuf, device="cuda")
    b = torch.as_tensor(bbuf, device="cuda")
    n = torch.as_tensor(nbuf, device="cuda").view(torch.int16)
    assert torch.equal(w.cpu(), rw) and torch.equal(b.cpu(), rb)
    ref_experts = [synth.to_device(t, "cuda") for t in experts]
    ref_bank = rt.create_bank(ref_experts)
    for tokens in (8, 300):
        x = synth.activations(tokens, HID, 17 + tokens, "cuda")
        got = rt.moe_layer(x, w, b, bank, want_routes=True)
        ref = rt.moe_layer(x, rw.cuda(), rb.cuda(), ref_bank, want_routes=True)
        assert torch.equal(got.selected, ref.selected)
        assert torch.equal(got.output, ref.output), f"T{tokens}"
        blk = rt.moe_block(x, n, 1e-5, w, b, bank)
        blk_ref = rt.moe_block(x, nw.cuda(), 1e-5, rw.cuda(), rb.cuda(), ref_bank)
        assert torch.equal(blk.output, blk_ref.output)
    for buf in (wbuf, bbuf, nbuf):
        buf.free()
    for f in files:
        f.close()


def test_bank_from_expert_containers(rt, tmp_path):
    # one PWEXPRT1 container per expert (docs/EXPERT_CONTAINER.md: bounded
    # expert streaming), repacked from the shards, loads into the same bank
    from mimo_prismwing_b200 import checkpoint as C
    from mimo_prismwing_b200 import synth
    paths, experts, (rw, rb, _) = _checkpoint(tmp_path)
    containers = []
    for e in range(E):
        names = [f"model.layers.{LAYER}.mlp.experts.{e}.{p}.weight{s}"
                 for p in ("gate_proj", "up_proj", "down_proj") for s in ("", "_scale_inv")]
        out = str(tmp_path / f"layer{LAYER}-expert{e}.pwexpert")
        containers.append(C.repack_expert_container(paths[e // 8], out, names))
    bank = C.load_bank(rt, containers, LAYER, 0, E)
    ref_bank = rt.create_bank([synth.to_device(t, "cuda") for t in experts])
    x = synth.activations(8, HID, 5, "cuda")
    got = rt.moe_layer(x, rw.cuda(), rb.cuda(), bank)
    ref = rt.moe_layer(x, rw.cuda(), rb.cuda(), ref_bank)
    assert torch.equal(got.output, ref.output)
    for c in containers:
        c.close()


def test_bank_load_fails_closed(rt, tmp_path):
    from mimo_prismwing_b200 import checkpoint as C
    paths, _, _ = _checkpoint(tmp_path, bad_byte=True)
    files = [C.MappedSafetensors.open(p) for p in paths]
    free0, _ = torch.cuda.mem_get_info()
    with pytest.raises(C.CheckpointError) as e:  # a NaN byte (0x7f) in expert 11's up projection
        C.load_bank(rt, files, LAYER, 0, E)
    assert e.value.status == -3 and "11" in str(e.value)
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info()[0] >= free0 - (2 << 20)  # the upload was released
    with pytest.raises(C.CheckpointError) as e:  # experts 16.. do not exist
        C.load_bank(rt, files, LAYER, 8, 9)
    assert e.value.status == -10 and "absent" in str(e.value)
    with pytest.raises(C.CheckpointError) as e:  # the same shard twice: every tensor is ambiguous
        C.load_bank(rt, [files[0], files[0]], LAYER, 0, 1)
    assert e.value.status == -10 and "more than one file" in str(e.value)
    with pytest.raises(C.CheckpointError) as e:  # dtype / shape checks of pw_tensor_upload
        C.upload(rt, files, f"model.layers.{LAYER}.mlp.gate.weight", "BF16")
    assert e.value.status == -2
    for f in files:
        f.close()
