"""Host logic of the fused row-parallel layer without a GPU: ``tp_linear.install()`` rebinds
RowParallelLinear.forward and keeps the original forward for every layer the kernel does not
cover (bf16 weights, a bias, tensor-parallel size 1, more rows than the buffers hold)."""
import types

import torch


class _FakeRowParallel:
    """Stand-in for nanovllm.layers.linear.RowParallelLinear: only what the rebinding reads."""

    def __init__(self, quantized=True, tp_size=2, bias=None):
        self.quantized, self.tp_size, self.bias = quantized, tp_size, bias
        self.weight = torch.zeros(256, 128)
        self.weight_scale = None

    def forward(self, x):
        return ("original", x.shape[0])


def test_install_keeps_the_original_forward_where_the_kernel_does_not_apply():
    from nanovllm_b200 import tp_linear
    module = types.SimpleNamespace(RowParallelLinear=_FakeRowParallel)
    orig = tp_linear.install(module, max_tokens=64)
    try:
        assert orig is not _FakeRowParallel.forward
        x = torch.zeros(8, 128)
        for layer in (_FakeRowParallel(quantized=False), _FakeRowParallel(tp_size=1),
                      _FakeRowParallel(bias=torch.zeros(256))):
            assert layer.forward(x) == ("original", 8)
        assert _FakeRowParallel().forward(torch.zeros(65, 128)) == ("original", 65)
    finally:
        _FakeRowParallel.forward = orig
    assert _FakeRowParallel().forward(torch.zeros(3, 128)) == ("original", 3)
