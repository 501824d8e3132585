"""The vLLM boundary: registration, parameter contract, weight loading (CPU) and apply (GPU)."""
import pytest
import torch


def test_param_shapes_match_reference_contract():
    from vq2_vllm.plugin import param_shapes
    s = param_shapes(256, 4096, 2048)
    assert s["w13_lo"] == ((256, 4096, 1024), torch.uint8)
    assert s["w13_hi"] == ((256, 4096, 256), torch.uint8)
    assert s["w13_sc"] == ((256, 4096, 64), torch.float16)
    assert s["w2_lo"] == ((256, 4096, 512), torch.uint8)
    assert s["w2_sc"] == ((256, 4096, 32), torch.float16)
    assert s["w13_cb"] == ((1024, 4), torch.float16)


def test_weight_loader_places_gate_and_up_halves():
    from vq2_vllm.plugin import weight_loader
    p = torch.nn.Parameter(torch.zeros(2, 8, 4, dtype=torch.uint8), requires_grad=False)
    weight_loader(p, torch.full((4, 4), 1, dtype=torch.uint8), "w13_lo", "w1", 1)
    weight_loader(p, torch.full((4, 4), 3, dtype=torch.uint8), "w13_lo", "w3", 1)
    assert p[1, :4].eq(1).all() and p[1, 4:].eq(3).all() and p[0].eq(0).all()
    cb = torch.nn.Parameter(torch.zeros(1024, 4, dtype=torch.float16), requires_grad=False)
    weight_loader(cb, torch.ones(1024, 4), "w13_cb", None, None)
    assert cb.eq(1).all()


def test_register_with_vllm():
    pytest.importorskip("vllm")
    import vq2_vllm
    from vllm.model_executor.layers.quantization import get_quantization_config
    cls = vq2_vllm.register()
    assert get_quantization_config("vq2") is cls
    cfg = cls.from_config({"quant_method": "vq2", "vdim": 4, "k": 1024, "group": 64})
    assert cfg.get_name() == "vq2" and cfg.group == 64
    with pytest.raises(ValueError):
        cls.from_config({"vdim": 8})


def test_bare_module_names_resolve():
    import sys

    import vq2_vllm  # noqa: F401
    assert hasattr(sys.modules["vq2_kernel"], "vq2_moe_fused_10b")
    assert hasattr(sys.modules["moe_align"], "moe_align")


@pytest.mark.gpu
@pytest.mark.parametrize("N", [3, 300])
def test_apply_dispatch_matches_oracle(N):
    """apply(): decode kernel below VQ2_WMMA_MIN tokens, grouped GEMM at or above (fp8 default)."""
    from types import SimpleNamespace

    from oracle import torch_ref
    from vq2_vllm import synth
    from vq2_vllm.plugin import apply_moe
    L = synth.make_layer(16, 1024, 512, seed=0, device="cuda")
    layer = SimpleNamespace(**L)
    x = synth.make_tokens(N, 1024, seed=1, device="cuda")
    ids, w = synth.route_uniform(N, 16, 8, seed=2, device="cuda")
    out = apply_moe(layer, x, w, ids)
    assert out.dtype == x.dtype
    ref = torch_ref.moe_ref(x, ids, w, L) if N < 256 else torch_ref.moe_prefill_fp8_ref(x, ids, w, L)
    assert torch_ref.rel_l2(out.float(), ref) < 3e-2


def test_fused_layer_file_sharded_read(tmp_path):
    """An expert-parallel rank reads only its experts of a fused layer file (slices), identical to
    slicing the whole layer."""
    from safetensors.torch import save_file
    from vq2_vllm import ep, synth
    from vq2_vllm.plugin import read_fused_layer
    layer = synth.make_layer(8, 256, 128, seed=3)
    path = str(tmp_path / "experts_fused_layer_0.safetensors")
    save_file({k: v.contiguous() for k, v in layer.items()}, path)
    whole = read_fused_layer(path)
    for k in layer:
        assert torch.equal(whole[k], layer[k])
    for rank in range(4):
        mine = ep.load_local_layer(path, rank, 4)
        ref = ep.local_layer(layer, rank, 4)
        for k in layer:
            assert torch.equal(mine[k], ref[k]), (rank, k)
        assert mine["w13_lo"].shape[0] == 2 and mine["w13_cb"].shape == (1024, 4)


@pytest.mark.gpu
@pytest.mark.parametrize("N", [4, 300])
def test_fused_layer_file_to_device_then_apply(tmp_path, N):
    """Row f3 on the device: a fused layer file on disk, an expert-parallel rank's layer whose
    parameters live on the GPU, the post-load hook reading only that rank's experts onto it, then
    apply() on global expert ids — against the oracle over the same expert window."""
    from types import SimpleNamespace

    from safetensors.torch import save_file

    from oracle import torch_ref
    from vq2_vllm import synth
    from vq2_vllm.plugin import apply_moe, param_shapes, process_weights_after_loading
    E, H, I, world, rank = 16, 1024, 512, 4, 2
    full = synth.make_layer(E, H, I, seed=5)
    save_file({k: v.contiguous() for k, v in full.items()}, str(tmp_path / "experts_fused_layer_3.safetensors"))
    per = E // world
    params = {k: torch.empty(*shape, dtype=dt, device="cuda") for k, (shape, dt) in param_shapes(per, H, I).items()}
    layer = SimpleNamespace(layer_name="model.layers.3.mlp.experts", local_num_experts=per, ep_rank=rank,
                            **{k: torch.nn.Parameter(v, requires_grad=False) for k, v in params.items()})
    assert process_weights_after_loading(layer, directory=str(tmp_path))
    assert layer.vq2_expert_base == rank * per
    for k, v in full.items():
        want = v if k.endswith("cb") else v[rank * per:(rank + 1) * per]
        assert torch.equal(getattr(layer, k).cpu(), want), k
    x = synth.make_tokens(N, H, seed=6, device="cuda")
    ids, w = synth.route_uniform(N, E, 8, seed=7, device="cuda")
    out = apply_moe(layer, x, w, ids).float()
    Lc = {k: v.cuda() for k, v in full.items()}
    win = {k: (v if k.endswith("cb") else v[rank * per:(rank + 1) * per]) for k, v in Lc.items()}
    f = torch_ref.moe_ref if N < 256 else torch_ref.moe_prefill_fp8_ref
    ref = f(x, ids, w, win, expert_base=rank * per)
    assert torch_ref.rel_l2(out, ref) < 3e-2
    other = SimpleNamespace(layer_name="model.layers.9.mlp.experts", **params)
    assert not process_weights_after_loading(other, directory=str(tmp_path))   # no file: nothing read
