"""The PEFT adapter directory written and read by the C++ host library (r97host_adapter_write / _read) on
CPU: the reference's own golden adapter fixture (tests/golden/adapter_ref, the reference's
tests/fixtures/adapter_ref) reproduced byte for byte and read back exactly; bf16, non-integral alpha and a
transformed-trunk basis round-trip; the file loads with the safetensors library; bad reads are refused."""
import json
import os

import numpy as np
import pytest
import torch

from r97training_b200 import peft

GOLD = os.path.join(os.path.dirname(__file__), "golden", "adapter_ref")
MODULE = "model.layers.0.mlp.down_proj"
NAMES = [MODULE + ".lora_A", MODULE + ".lora_B"]
SHAPES = [(2, 256), (128, 2)]


def _golden_values():
    a = np.array([r * 256 + k for r in range(2) for k in range(256)], dtype=np.float32)
    b = np.array([-(n * 2 + r + 1) for n in range(128) for r in range(2)], dtype=np.float32)
    return np.concatenate([a, b])


def test_writer_reproduces_the_reference_fixture(tmp_path):
    out = str(tmp_path / "adapter")
    peft.write(out, NAMES, SHAPES, _golden_values(), base_model="qwen3.5-tiny", rank=2, alpha=4.0,
               targets=["down_proj"])
    for f in ("adapter_config.json", "adapter_model.safetensors"):
        assert open(os.path.join(out, f), "rb").read() == open(os.path.join(GOLD, f), "rb").read(), f


def test_reader_reads_the_reference_fixture():
    vals, rank, alpha, dt = peft.read(GOLD, NAMES, SHAPES)
    assert (rank, alpha, dt) == (2, 4.0, "f32")
    assert np.array_equal(vals, _golden_values())


def test_bf16_round_trip_and_safetensors_interop(tmp_path):
    rs = np.random.RandomState(0)
    names = ["model.layers.3.self_attn.q_proj.lora_A", "model.layers.3.self_attn.q_proj.lora_B",
             "model.layers.0.linear_attn.in_proj_qkvz.lora_A", "model.layers.0.linear_attn.in_proj_qkvz.lora_B"]
    shapes = [(8, 64), (96, 8), (8, 64), (128, 8)]
    vals = rs.normal(size=sum(r * c for r, c in shapes)).astype(np.float32)
    out = str(tmp_path / "a")
    peft.write(out, names, shapes, vals, base_model='m"odel\\x', rank=8, alpha=2.5,
               targets=["q_proj", "in_proj_qkvz"], dtype="bf16", input_basis="fwht128")
    cfg = json.load(open(os.path.join(out, "adapter_config.json")))
    assert cfg["lora_alpha"] == 2.5 and cfg["r"] == 8 and cfg["radiance_input_basis"] == "fwht128"
    assert cfg["base_model_name_or_path"] == 'm"odel\\x' and list(cfg)[0] == "peft_type"
    back, rank, alpha, dt = peft.read(out, names, shapes)
    assert (rank, alpha, dt) == (8, 2.5, "bf16")
    want = torch.from_numpy(vals).bfloat16().float().numpy()
    assert np.array_equal(back, want)
    from safetensors.torch import load_file
    tensors = load_file(os.path.join(out, "adapter_model.safetensors"))
    assert sorted(tensors) == sorted("base_model.model." + n + ".weight" for n in names)
    off = 0
    for n, (r, c) in zip(names, shapes):
        t = tensors["base_model.model." + n + ".weight"]
        assert t.dtype == torch.bfloat16 and tuple(t.shape) == (r, c)
        assert np.array_equal(t.float().numpy().ravel(), want[off:off + r * c])
        off += r * c


def test_reader_refuses_mismatches(tmp_path):
    with pytest.raises(RuntimeError, match="shape mismatch"):
        peft.read(GOLD, NAMES, [(2, 256), (64, 2)])
    with pytest.raises(RuntimeError, match="no tensor"):
        peft.read(GOLD, [MODULE + ".lora_A", "model.layers.1.mlp.down_proj.lora_B"], SHAPES)
    with pytest.raises(RuntimeError, match="does not name"):
        peft.read(GOLD, NAMES[:1], SHAPES[:1])
    with pytest.raises(RuntimeError, match="cannot open"):
        peft.read(str(tmp_path / "missing"), NAMES, SHAPES)
