"""Real-weight ingestion (checkpoint state_dict keys + Pangu_Clusters files -> TauSparseMoE):
CPU tests of the key mapping, the cluster-file format and the physical reorder; one GPU test
runs ingested layers at the reference's shipped configuration (E=192, G=32) through decode
and prefill against the oracle."""
import numpy as np
import pytest
import torch

from conftest import assert_close_out, oracle, pkg
from gpu_helpers import check_against_oracle, run_decode

PREFIX = "model.model.layers"


def _state_dict(layers, masks_as_buffer=True):
    """The keys ``CustomOpenPangu.state_dict()`` has for the MoE MLP of each layer
    (src/openpangu_moe.py:58-62, src/MoEBlock.py:125-143)."""
    sd = {}
    for i, L in enumerate(layers):
        b = f"{PREFIX}.{i}.mlp."
        sd[b + "gate_proj.weight"] = L.gate_w
        sd[b + "up_proj.weight"] = L.up_w
        sd[b + "down_proj.weight"] = L.down_w
        sd[b + "moelayer.mlp_router.0.weight"] = L.router_w
        if masks_as_buffer:  # registered with the router's dtype (src/MoEBlock.py:143)
            sd[b + "moelayer.experts_masks"] = torch.nn.functional.one_hot(L.experts_id, L.experts).t().to(torch.bfloat16)
        sd[b + "moelayer.activated_statistics"] = torch.zeros(L.experts, dtype=torch.long)
        sd[f"{PREFIX}.{i}.self_attn.q_proj.weight"] = torch.zeros(2, 2)  # unrelated keys are ignored
    return sd


def _layers(golden, n=2):
    """Layers at E=192, G=32 whose first uses the reference's real layer-0 cluster assignment."""
    synth = pkg().synth
    case = next(c for c in golden["cases"] if c["name"].startswith("pangu_e192"))
    out = []
    for i in range(n):
        L = synth.make_layer(40 + i, 256, 192, 32, router_scale=1.75)
        if i == 0:
            L.experts_id = case["experts_id"].long()
        out.append(L)
    return out


def test_cluster_file_format(tmp_path, golden):
    """Files in the reference's format (np.savetxt floats, one id per neuron) parse to ids."""
    ing = pkg().ingest
    ids = next(c for c in golden["cases"] if c["name"].startswith("pangu_e192"))["experts_id"].long()
    p = tmp_path / "layer_0_k32.txt"
    np.savetxt(p, ids.numpy().astype(np.float64))
    assert torch.equal(ing.load_cluster_ids(str(p)), ids)
    m = ing.masks_from_ids(ids, 192)
    assert m.shape == (192, 6144) and torch.equal(m.sum(0), torch.ones(6144, dtype=torch.long))
    bad = tmp_path / "bad.txt"
    np.savetxt(bad, np.array([0.0, 1.5]))
    with pytest.raises(ValueError):
        ing.load_cluster_ids(str(bad))


@pytest.mark.parametrize("masks_as_buffer", [True, False])
def test_state_dict_to_reordered_buffers(tmp_path, golden, masks_as_buffer):
    ing = pkg().ingest
    layers = _layers(golden)
    sd = _state_dict(layers, masks_as_buffer)
    cdir = None
    if not masks_as_buffer:
        for i, L in enumerate(layers):
            np.savetxt(tmp_path / f"layer_{i}_k32.txt", L.experts_id.numpy().astype(np.float64))
        cdir = str(tmp_path)
    assert ing.layer_indices(sd) == [0, 1]
    mods = ing.moe_layers_from_state_dict(sd, group_size=32, tau=0.7, device="cpu", cluster_dir=cdir)
    for i, L in enumerate(layers):
        Wg, Wu, Wd, R = oracle().reference_layout(L)
        m = mods[i]
        assert m.tau == 0.7 and (m.hidden_size, m.num_experts, m.group_size) == (256, 192, 32)
        assert torch.equal(m.W_gate, Wg) and torch.equal(m.W_up, Wu)
        assert torch.equal(m.W_down, Wd) and torch.equal(m.router, R)
    # a checkpoint saved after the reorder: tau_moe buffers mount as they are
    post = {}
    for i, m in mods.items():
        for n in ("W_gate", "W_up", "W_down", "router"):
            post[f"{PREFIX}.{i}.mlp.tau_moe.{n}"] = getattr(m, n).clone()
    mods2 = ing.moe_layers_from_state_dict(post, group_size=32, tau=0.7, device="cpu")
    for i in mods:
        for n in ("W_gate", "W_up", "W_down", "router"):
            assert torch.equal(getattr(mods2[i], n), getattr(mods[i], n))


def test_state_dict_missing_pieces(golden):
    ing = pkg().ingest
    sd = _state_dict(_layers(golden, 1), masks_as_buffer=False)
    with pytest.raises(KeyError):
        ing.moe_layers_from_state_dict(sd, group_size=32, tau=0.7, device="cpu")  # no masks, no files
    del sd[f"{PREFIX}.0.mlp.up_proj.weight"]
    with pytest.raises(KeyError, match="up_proj"):
        ing.moe_layers_from_state_dict(sd, group_size=32, tau=0.7, device="cpu", cluster_dir="/nonexistent")
    with pytest.raises(ValueError):
        ing.moe_layers_from_state_dict(_state_dict(_layers(golden, 1)), group_size=64, tau=0.7, device="cpu")


@pytest.mark.gpu
def test_ingested_layers_on_gpu(golden, cuda):
    """Ingested E=192/G=32 layers (real layer-0 cluster assignment) through decode and prefill."""
    ing, synth = pkg().ingest, pkg().synth
    layers = _layers(golden)
    mods = ing.moe_layers_from_state_dict(_state_dict(layers), group_size=32, tau=0.7, device=cuda)
    for i, L in enumerate(layers):
        x = synth.make_tokens(60 + i, 3, 256)
        out, lg, w = run_decode(mods[i], x, cuda)
        check_against_oracle(L, x, 0.7, out, lg, w, what=f"ingested decode layer {i}")
        xp = synth.make_tokens(70 + i, 200, 256)
        lgp = torch.empty(200, 192, dtype=torch.bfloat16, device=cuda)
        y = mods[i].forward_prefill(xp.to(cuda), logits_out=lgp)
        mods[i].check_device_status()
        tf = oracle().moe_mlp(xp, L, 0.7, logits=lgp.cpu())
        assert_close_out(y.cpu(), tf.out, f"ingested prefill layer {i}")
