"""The drop-in op namespace on the CPU: ``torch.ops.mini_vllm_ops`` carries the reference's 15
schemas (``csrc/bindings/ops_binding.cpp:11-25``) verbatim plus the decode ops, and none of them
has a CPU implementation: a CPU tensor raises instead of falling back to host math."""
import pytest
import torch

from llm_pytorch_inference_b200 import torch_ops


def _registered(name):
    return str(getattr(torch.ops.mini_vllm_ops, name).default._schema)


def test_namespace_holds_every_schema_verbatim():
    assert torch_ops.register()
    assert len(torch_ops.REFERENCE_SCHEMAS) == 15
    for schema in torch_ops.REFERENCE_SCHEMAS + torch_ops.DECODE_SCHEMAS:
        name = schema.split("(")[0]
        assert _registered(name) == f"{torch_ops.NAMESPACE}::{schema}", name
    assert set(torch_ops.IMPLS) == {s.split("(")[0] for s in torch_ops.REFERENCE_SCHEMAS + torch_ops.DECODE_SCHEMAS}


def test_register_is_idempotent():
    assert torch_ops.register() and torch_ops.register()


@pytest.mark.parametrize("call", [
    lambda: torch.ops.mini_vllm_ops.rmsnorm_forward(torch.ones(2, 8), torch.ones(8), 1e-6),
    lambda: torch.ops.mini_vllm_ops.silu_forward(torch.ones(4)),
    lambda: torch.ops.mini_vllm_ops.greedy_sample(torch.ones(2, 16)),
    lambda: torch.ops.mini_vllm_ops.softmax_forward(torch.ones(2, 16)),
])
def test_cpu_tensors_have_no_kernel(call):
    with pytest.raises((NotImplementedError, RuntimeError)):
        call()
