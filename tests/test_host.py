"""Host logic of the drop-in on the CPU: the reference's refusals (src/macai/gated_delta/op.py:124-131, :270-273;
tests/test_harness.py:169-173), shape checks, the absence of any CPU path, and install() routing transformers'
Qwen3.5-family modules (and already-built layers) to this package's rule (src/macai/patch.py:27-98)."""
import importlib

import pytest
import torch

from macai_b200 import patch
from macai_b200.gated_delta import chunk_gated_delta_rule, l2norm, op, recurrent_reference


def test_packed_rows_checked_before_any_launch():
    """cu_seqlens (which the reference refuses, op.py:270-273) is taken with fla's semantics; wrong boundary lists,
    a batch size other than 1 and a per-sequence initial state of the wrong shape are refused on the host, and there
    is still no CPU path."""
    x = torch.zeros(1, 4, 1, 128, dtype=torch.bfloat16)
    for bad in ([0, 2, 3], [1, 2, 4], [0, 3, 2, 4], [4], [[0, 4]]):
        with pytest.raises(ValueError):
            chunk_gated_delta_rule(x, x, x, x[..., 0], x[..., 0], cu_seqlens=torch.tensor(bad))
    x2 = torch.zeros(2, 4, 1, 128, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="batch size must be 1"):
        chunk_gated_delta_rule(x2, x2, x2, x2[..., 0], x2[..., 0], cu_seqlens=torch.tensor([0, 2, 4]))
    with pytest.raises(ValueError, match="initial_state"):
        chunk_gated_delta_rule(x, x, x, x[..., 0], x[..., 0], cu_seqlens=torch.tensor([0, 2, 4]),
                               initial_state=torch.zeros(1, 1, 128, 128, dtype=torch.bfloat16))
    with pytest.raises(RuntimeError, match="CUDA"):
        chunk_gated_delta_rule(x, x, x, x[..., 0], x[..., 0], cu_seqlens=torch.tensor([0, 2, 4]))


def test_unsupported_head_width_refused():
    """Widths above the built 128 are refused (NotImplementedError), widths that are not multiples of 32 rejected
    (ValueError, as the reference's op.py:124-125); 32-96 are padded (tests/test_gpu_head_widths.py)."""
    x = torch.zeros(1, 4, 1, 256, dtype=torch.bfloat16)
    with pytest.raises(NotImplementedError):
        chunk_gated_delta_rule(x, x, x, x[..., 0], x[..., 0])
    x = torch.zeros(1, 4, 1, 80, dtype=torch.bfloat16)
    with pytest.raises(ValueError):
        chunk_gated_delta_rule(x, x, x, x[..., 0], x[..., 0])


def test_shape_errors():
    q = torch.zeros(1, 4, 2, 128, dtype=torch.bfloat16)
    v = torch.zeros(1, 4, 3, 128, dtype=torch.bfloat16)
    with pytest.raises(ValueError):
        chunk_gated_delta_rule(q, q, v, v[..., 0], v[..., 0])               # 3 value heads, 2 key heads
    v = torch.zeros(1, 4, 2, 128, dtype=torch.bfloat16)
    with pytest.raises(ValueError):
        chunk_gated_delta_rule(q, q, v, v[..., 0, 0], v[..., 0])             # g of the wrong shape


def test_no_cpu_path():
    x = torch.zeros(1, 4, 1, 128, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="CUDA"):
        chunk_gated_delta_rule(x, x, x, x[..., 0], x[..., 0])


def test_reference_utilities_match_oracle():
    from oracle import gated_delta_f64 as ref
    gen = torch.Generator().manual_seed(0)
    q = l2norm(torch.randn(1, 9, 2, 8, generator=gen, dtype=torch.float64)) * 8 ** -0.5
    k = l2norm(torch.randn(1, 9, 2, 8, generator=gen, dtype=torch.float64))
    v = torch.randn(1, 9, 2, 8, generator=gen, dtype=torch.float64)
    g, b = -torch.rand(1, 9, 2, generator=gen, dtype=torch.float64), torch.rand(1, 9, 2, generator=gen, dtype=torch.float64)
    s0 = torch.randn(1, 2, 8, 8, generator=gen, dtype=torch.float64)
    o1, s1 = recurrent_reference(q, k, v, g, b, s0)
    o2, s2 = ref.recurrence(q, k, v, g, b, s0)
    assert torch.equal(o1, o2) and torch.equal(s1, s2)


def test_install_routes_transformers():
    mod = importlib.import_module("transformers.models.qwen3_5.modeling_qwen3_5")
    before = mod.torch_chunk_gated_delta_rule
    with patch.installed():
        assert mod.torch_chunk_gated_delta_rule is chunk_gated_delta_rule
        # transformers 5.x binds `chunk_gated_delta_rule or torch_chunk_gated_delta_rule` in the layer's __init__
        assert mod.chunk_gated_delta_rule is chunk_gated_delta_rule
        assert ("transformers.models.qwen3_5.modeling_qwen3_5", "torch_chunk_gated_delta_rule") in patch.patched()
    assert mod.torch_chunk_gated_delta_rule is before
    assert not patch.patched()


def test_install_rebinds_built_layers():
    class Layer(torch.nn.Module):
        def __init__(self):
            super().__init__()
            self.chunk_gated_delta_rule = lambda *a, **k: "original"

    model = torch.nn.Sequential(Layer(), Layer())
    with patch.installed(model=model):
        assert all(m.chunk_gated_delta_rule is chunk_gated_delta_rule for m in model)
    assert all(m.chunk_gated_delta_rule() == "original" for m in model)


def test_qwen3_5_layer_binds_patched_rule():
    """A Qwen3.5 linear-attention layer built after install() calls this package's rule."""
    mod = importlib.import_module("transformers.models.qwen3_5.modeling_qwen3_5")
    from transformers.models.qwen3_5.configuration_qwen3_5 import Qwen3_5TextConfig
    cfg = Qwen3_5TextConfig(hidden_size=64, num_attention_heads=2, num_key_value_heads=1, head_dim=32,
                            linear_num_key_heads=2, linear_num_value_heads=2, linear_key_head_dim=128,
                            linear_value_head_dim=128, linear_conv_kernel_dim=4, num_hidden_layers=1,
                            intermediate_size=64, vocab_size=32)
    with patch.installed():
        layer = mod.Qwen3_5GatedDeltaNet(cfg, layer_idx=0) if torch.cuda.is_available() else None
        if layer is None:
            pytest.skip("the layer's constructor places a module on the current CUDA device")
        assert layer.chunk_gated_delta_rule is chunk_gated_delta_rule


def test_wide_query_dtypes_refused_by_default(monkeypatch):
    """fp16 / fp32 queries: NotImplementedError before any launch unless op.ALLOW_BF16_COMPUTE (the kernels' bf16
    operands miss those dtypes' accuracy); other dtypes: TypeError."""
    import torch
    from macai_b200.gated_delta import chunk_gated_delta_rule, op
    for dt in (torch.float16, torch.float32):
        x = torch.zeros(1, 4, 1, 128, dtype=dt)
        with pytest.raises(NotImplementedError, match="ALLOW_BF16_COMPUTE"):
            chunk_gated_delta_rule(x, x, x, x[..., 0].float(), x[..., 0].float())
    with pytest.raises(TypeError):
        x = torch.zeros(1, 4, 1, 128, dtype=torch.float64)
        chunk_gated_delta_rule(x, x, x, x[..., 0], x[..., 0])
    monkeypatch.setattr(op, "ALLOW_BF16_COMPUTE", True)
    x = torch.zeros(1, 4, 1, 128, dtype=torch.float32)
    with pytest.raises(RuntimeError, match="no CPU path"):   # past the dtype check: only the device is wrong now
        chunk_gated_delta_rule(x, x, x, x[..., 0], x[..., 0])
