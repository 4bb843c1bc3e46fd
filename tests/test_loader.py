"""The checkpoint loader (senmoe.loader) on synthetic MLX safetensors
checkpoints written with the reference's tensor names and config keys
(src/engine/mlx_native.rs:3365-3530 DeepSeek-V2, :3090-3357 Gemma-4):
shard index, the mlp.* / moe.* spellings, first_k_dense_replace,
the language_model. prefix, text_config, per-module router quantization."""
import json
import os
import struct

import numpy as np
import pytest

from oracle import oracle as O

torch = pytest.importorskip("torch")


def write_safetensors(path, tensors):
    """Minimal safetensors writer: {name: (dtype code, array)}."""
    head, blobs, off = {}, [], 0
    for name, (code, a) in tensors.items():
        b = np.ascontiguousarray(a).tobytes()
        head[name] = {"dtype": code, "shape": list(a.shape), "data_offsets": [off, off + len(b)]}
        blobs.append(b)
        off += len(b)
    h = json.dumps(head).encode()
    h += b" " * ((8 - len(h) % 8) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for b in blobs:
            f.write(b)


def deepseek_checkpoint(tmp, cfg, mw1, mw2):
    """3 layers: layer 0 dense, layers 1 (mlp.* names) and 2 (moe.* names) MoE;
    two shards and an index."""
    def layer(i, mw, sp):
        p = f"model.layers.{i}.{sp}"
        t = {f"{p}.gate.weight": ("BF16", mw.router_w)}
        for n in ("gate", "up", "down"):
            t[f"{p}.switch_mlp.{n}_proj.weight"] = ("U32", getattr(mw, f"{n}_w"))
            t[f"{p}.switch_mlp.{n}_proj.scales"] = ("BF16", getattr(mw, f"{n}_s"))
            t[f"{p}.switch_mlp.{n}_proj.biases"] = ("BF16", getattr(mw, f"{n}_b"))
            t[f"{p}.shared_experts.{n}_proj.weight"] = ("U32", getattr(mw, f"sh_{n}_w"))
            t[f"{p}.shared_experts.{n}_proj.scales"] = ("BF16", getattr(mw, f"sh_{n}_s"))
            t[f"{p}.shared_experts.{n}_proj.biases"] = ("BF16", getattr(mw, f"sh_{n}_b"))
        return t
    s0 = {"model.layers.0.mlp.gate_proj.weight": ("U32", np.zeros((4, 4), np.uint32))}
    s0.update(layer(1, mw1, "mlp"))
    s1 = layer(2, mw2, "moe")
    write_safetensors(os.path.join(tmp, "model-00001-of-00002.safetensors"), s0)
    write_safetensors(os.path.join(tmp, "model-00002-of-00002.safetensors"), s1)
    wm = {k: "model-00001-of-00002.safetensors" for k in s0}
    wm.update({k: "model-00002-of-00002.safetensors" for k in s1})
    with open(os.path.join(tmp, "model.safetensors.index.json"), "w") as f:
        json.dump({"metadata": {}, "weight_map": wm}, f)
    with open(os.path.join(tmp, "config.json"), "w") as f:
        json.dump({"model_type": "deepseek_v2", "hidden_size": cfg.hidden, "num_hidden_layers": 3,
                   "moe_intermediate_size": cfg.intermediate, "n_routed_experts": cfg.num_experts,
                   "num_experts_per_tok": cfg.top_k, "n_shared_experts": 1, "first_k_dense_replace": 1,
                   "moe_layer_freq": 1, "norm_topk_prob": True, "routed_scaling_factor": 1.0,
                   "quantization": {"group_size": 64, "bits": cfg.bits}}, f)


def small_cfg(bits=4):
    return O.MoeConfig(hidden=128, intermediate=64, num_experts=8, top_k=2, bits=bits, shared_intermediate=64)


def test_deepseek_layers_and_tensors(tmp_path):
    from senmoe import loader
    cfg = small_cfg()
    mw1, mw2 = O.make_layer(cfg, seed=1), O.make_layer(cfg, seed=2)
    deepseek_checkpoint(str(tmp_path), cfg, mw1, mw2)
    got = loader.load_deepseek_moe(str(tmp_path), device="cpu")
    assert [g.layer for g in got] == [1, 2]
    for g, mw in zip(got, (mw1, mw2)):
        a = g.args
        assert (a.hidden_size, a.moe_intermediate_size, a.n_routed_experts, a.num_experts_per_tok,
                a.n_shared_experts, a.bits, a.group_size) == (128, 64, 8, 2, 1, 4, 64)
        w = g.weights
        np.testing.assert_array_equal(w.router_weight.view(torch.int16).numpy().view(np.uint16), mw.router_w)
        np.testing.assert_array_equal(w.gate_proj.weight.numpy().view(np.uint32), mw.gate_w)
        np.testing.assert_array_equal(w.down_proj.scales.view(torch.int16).numpy().view(np.uint16), mw.down_s)
        np.testing.assert_array_equal(w.shared_up_proj.biases.view(torch.int16).numpy().view(np.uint16), mw.sh_up_b)
    assert [g.layer for g in loader.load_deepseek_moe(str(tmp_path), device="cpu", layers=[2])] == [2]


def test_single_file_and_float_scales(tmp_path):
    """A single model.safetensors; fp32 scales / biases are converted to bf16."""
    from senmoe import loader
    cfg = small_cfg()
    mw = O.make_layer(cfg, seed=3)
    t = {"model.layers.0.mlp.gate.weight": ("BF16", mw.router_w)}
    for n in ("gate", "up", "down"):
        t[f"model.layers.0.mlp.switch_mlp.{n}_proj.weight"] = ("U32", getattr(mw, f"{n}_w"))
        t[f"model.layers.0.mlp.switch_mlp.{n}_proj.scales"] = ("F32", O.bf16_to_f32(getattr(mw, f"{n}_s")))
        t[f"model.layers.0.mlp.switch_mlp.{n}_proj.biases"] = ("F32", O.bf16_to_f32(getattr(mw, f"{n}_b")))
    write_safetensors(os.path.join(tmp_path, "model.safetensors"), t)
    with open(os.path.join(tmp_path, "config.json"), "w") as f:
        json.dump({"hidden_size": 128, "num_hidden_layers": 1, "moe_intermediate_size": 64, "n_routed_experts": 8,
                   "num_experts_per_tok": 2, "n_shared_experts": 0}, f)
    (g,) = loader.load_deepseek_moe(str(tmp_path), device="cpu")
    assert g.args.bits == 4 and g.args.group_size == 64 and g.weights.shared_up_proj is None
    np.testing.assert_array_equal(g.weights.up_proj.scales.view(torch.int16).numpy().view(np.uint16), mw.up_s)


def gemma_checkpoint(tmp, cfg, mw, rw, router_bits):
    t = {}
    p = "language_model.model.layers.1"
    for n in ("gate", "up", "down"):
        t[f"{p}.experts.switch_glu.{n}_proj.weight"] = ("U32", getattr(mw, f"{n}_w"))
        t[f"{p}.experts.switch_glu.{n}_proj.scales"] = ("BF16", getattr(mw, f"{n}_s"))
        t[f"{p}.experts.switch_glu.{n}_proj.biases"] = ("BF16", getattr(mw, f"{n}_b"))
    t[f"{p}.router.proj.weight"] = ("U32", rw.proj_w)
    t[f"{p}.router.proj.scales"] = ("BF16", rw.proj_s)
    t[f"{p}.router.proj.biases"] = ("BF16", rw.proj_b)
    t[f"{p}.router.scale"] = ("BF16", rw.scale)
    t[f"{p}.router.per_expert_scale"] = ("BF16", rw.per_expert_scale)
    t["language_model.model.layers.0.mlp.gate_proj.weight"] = ("U32", np.zeros((4, 4), np.uint32))
    write_safetensors(os.path.join(tmp, "model.safetensors"), t)
    with open(os.path.join(tmp, "config.json"), "w") as f:
        json.dump({"model_type": "gemma4",
                   "text_config": {"hidden_size": cfg.hidden, "num_hidden_layers": 2, "enable_moe_block": True,
                                   "num_experts": cfg.num_experts, "top_k_experts": cfg.top_k,
                                   "moe_intermediate_size": cfg.intermediate, "rms_norm_eps": 1e-6},
                   "quantization": {"group_size": 64, "bits": cfg.bits,
                                    "language_model.model.layers.1.router.proj": {"group_size": 64,
                                                                                  "bits": router_bits}}}, f)


def test_gemma_layers_and_tensors(tmp_path):
    from senmoe import loader
    cfg = O.MoeConfig(hidden=128, intermediate=64, num_experts=8, top_k=2, bits=4, activation=1)
    mw = O.make_layer(cfg, seed=5)
    rc = O.GemmaRouterConfig(hidden=128, num_experts=8, top_k=2, bits=8)
    rw = O.make_gemma_router(rc, seed=6)
    gemma_checkpoint(str(tmp_path), cfg, mw, rw, 8)
    (g,) = loader.load_gemma4_moe(str(tmp_path), device="cpu")
    assert g.layer == 1 and g.router_bits == 8 and g.rms_norm_eps == pytest.approx(1e-6)
    assert g.args.activation == 1 and g.args.num_experts_per_tok == 2 and g.weights.router_weight is None
    np.testing.assert_array_equal(g.weights.up_proj.weight.numpy().view(np.uint32), mw.up_w)
    np.testing.assert_array_equal(g.router.proj.weight.numpy().view(np.uint32), rw.proj_w)
    np.testing.assert_array_equal(g.router.per_expert_scale.view(torch.int16).numpy().view(np.uint16),
                                  rw.per_expert_scale)


def test_gemma_half_declared_moe_is_absent(tmp_path):
    from senmoe import loader
    with open(os.path.join(tmp_path, "config.json"), "w") as f:
        json.dump({"hidden_size": 128, "num_hidden_layers": 2, "enable_moe_block": True, "num_experts": 8}, f)
    write_safetensors(os.path.join(tmp_path, "model.safetensors"), {"x": ("U32", np.zeros(4, np.uint32))})
    assert loader.load_gemma4_moe(str(tmp_path), device="cpu") == []


def test_bad_tensor_size_is_rejected(tmp_path):
    from senmoe import loader
    path = os.path.join(tmp_path, "model.safetensors")
    write_safetensors(path, {"a": ("U32", np.zeros(4, np.uint32))})
    raw = bytearray(open(path, "rb").read())
    (n,) = struct.unpack("<Q", raw[:8])
    head = json.loads(raw[8:8 + n])
    head["a"]["shape"] = [5]
    h = json.dumps(head).encode()
    h += b" " * ((8 - len(h) % 8) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)) + h + bytes(raw[8 + n:]))
    ck = loader.SafetensorsCheckpoint(str(tmp_path))
    with pytest.raises(ValueError):
        ck.get("a")


def test_float_to_bf16_keeps_nan_and_scalar_tensors(tmp_path):
    """fp32 -> bf16 conversion rounds to nearest even and keeps every NaN a
    NaN of the same sign (a payload in the low mantissa bits must not round
    to Inf); a 0-d tensor reads back as a 0-d array."""
    from senmoe import loader
    bits = np.array([0x7F800001, 0xFF800001, 0x7FFFFFFF, 0xFFFFFFFF, 0x7FC00000, 0x3F808000, 0x3F818000,
                     0x7F7FFFFF, 0x00000001], np.uint32)
    f = bits.view(np.float32)
    write_safetensors(os.path.join(tmp_path, "model.safetensors"),
                      {"v": ("F32", f), "s": ("F32", np.array(2.5, np.float32))})
    ck = loader.SafetensorsCheckpoint(str(tmp_path))
    got = loader._bf16_bits(ck, "v")
    np.testing.assert_array_equal(got[:5], [0x7FC0, 0xFFC0, 0x7FC0, 0xFFC0, 0x7FC0])
    # 1.00390625 is a tie (rounds to even 1.0); 1.01171875 is a tie that rounds up
    np.testing.assert_array_equal(got[5:], [0x3F80, 0x3F82, 0x7F80, 0x0000])
    s = ck.get("s")
    assert s.shape == () and float(s) == 2.5
    assert loader._bf16_bits(ck, "s").shape == ()
