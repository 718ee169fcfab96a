"""BASELINE configs 3 and 5 (ResNet-50 and MobileNetV2 conv stacks) at batch 2: every layer, on
whatever kernel it dispatches to, equals the CPU oracle bit for bit (int8 requantized outputs)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import oracle

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("net", ["resnet50", "mobilenetv2"])
def test_network_layers_match_oracle(cuda_lib, net):
    import my_own_cnn_b200 as b2q
    from my_own_cnn_b200 import nets

    specs = nets.NETS[net]()
    data = nets.NetData(specs, batch=2, seed=42, device=torch.device("cuda"))
    paths = {}
    for i in range(len(specs)):
        data.run_layer(i)
        paths.setdefault(b2q.last_path(), []).append(specs[i].name)
    torch.cuda.synchronize()
    assert "cuda-core-generic" not in paths, paths.get("cuda-core-generic")
    for i, sp in enumerate(specs):
        x, w, b, s = nets.host_layer_tensors(sp, i, 42, 0, 2)
        np.testing.assert_array_equal(data.layers[i][1].cpu().numpy(), x, err_msg=f"{sp.name} input")
        a = oracle.conv_args(2, sp.h, sp.w, sp.c, sp.r, sp.r, sp.k, sp.pad, sp.pad, sp.stride, sp.stride, 1, 1,
                             sp.groups)
        acc = oracle.conv_s8(a, x, w, threads=2)
        e = sp.epilogue()
        ref = oracle.requant_s8(acc, b, s, e.zp_out, e.clamp_lo, e.clamp_hi)
        np.testing.assert_array_equal(data.layers[i][5].cpu().numpy(), ref, err_msg=sp.name)
