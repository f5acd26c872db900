"""Config 4: the 4-layer int8 MLP (MatMul -> Add bias -> Relu -> requantize to
uint8, x4, hidden 4096, batch 8192).  Every layer is one pfrt_qlinear launch
with bias, ReLU and requantization fused in its epilogue; the oracle composes
quant_ops.cpp:387-506 (accumulate, scale), math.cpp:222-226 (bias add),
activation.cpp:45-60 (ReLU) and quant_ops.cpp:15-127 (requantize) per layer.
Outputs must be bit-exact at every layer."""
import numpy as np
import pytest
import torch

import pyflamert_b200 as pf
from oracle import pyoracle as po
from pyflamert_b200 import sharding
from pyflamert_b200 import workloads as wl

pytestmark = pytest.mark.gpu


def run_layers(ctx, x, layers):
    ws = [(pf.QWeight(ctx, L.w, L.w_scale), torch.from_numpy(L.bias).cuda()) for L in layers]
    a = torch.from_numpy(np.ascontiguousarray(x)).cuda()
    outs = []
    for L, (w, b) in zip(layers, ws):
        a = w(a, L.a_scale, L.a_zp, bias=b, relu=True, out="uint8", y_scale=L.y_scale)
        outs.append(a)
    ctx.check()
    res = [o.cpu().numpy() for o in outs]
    for w, _ in ws:
        w.close()
    return res


def oracle_layers(x, layers):
    outs = []
    a = x
    for L in layers:
        a = po.qlinear(a, L.a_scale, L.a_zp, L.w, L.w_scale, bias=L.bias, relu=True, out="uint8",
                       y_scale=L.y_scale, y_zp=0)
        outs.append(a)
    return outs


def test_config4_full_batch_row_sample(ctx):
    """The whole 8192-row batch on the GPU; 12 rows followed through the oracle
    layer by layer (the layers are row-independent)."""
    x, layers = wl.mlp_case()
    got = run_layers(ctx, x, layers)
    rows = np.r_[0:4, 4094:4098, 8188:8192]
    ref = oracle_layers(x[rows], layers)
    for l in range(len(layers)):
        np.testing.assert_array_equal(got[l][rows], ref[l], err_msg=f"layer {l}")
    # the network stays alive to the last layer (not all-zero or all-saturated)
    last = got[-1]
    assert 0.05 < (last > 0).mean() < 0.95
    assert (last == 255).mean() < 0.5


@pytest.mark.parametrize("world", [2, 8])
def test_config4_batch_shards_equal_full_batch(ctx, world):
    """Batch sharding (what each rank runs at N GPUs) gives the full-batch rows."""
    x, layers = wl.mlp_case(batch=1024)
    full = run_layers(ctx, x, layers)[-1]
    for r in range(world):
        m0, m1 = sharding.batch_slice(x.shape[0], r, world)
        part = run_layers(ctx, x[m0:m1], layers)[-1]
        np.testing.assert_array_equal(part, full[m0:m1])
    ref = oracle_layers(x[:4], layers)[-1]
    np.testing.assert_array_equal(full[:4], ref)
