"""The prepared-weights cache (af2_set_weight_cache): the role of the reference's packing
cache per weights object (src/evoformer/block.ts:1310-1333).  With it on, a repeated call
with the same weights skips the preparation kernels and gives the same bits as an uncached
call; clearing it makes changed weights take effect."""
import numpy as np
import pytest

import af2cuda
import oracle
from helpers import pack, triangle_case

pytestmark = pytest.mark.gpu


def _attention_packed(rng, c=128, heads=4):
    def mat(i, o):
        return (rng.standard_normal((i, o)) / np.sqrt(i)).astype(np.float32).ravel()
    return np.concatenate([np.ones(c), np.zeros(c), mat(c, c), mat(c, c), mat(c, c), mat(c, c),
                           0.1 * rng.standard_normal(c), mat(c, c), np.zeros(c), mat(c, heads)]).astype(np.float32)


def _ops(device, torch, rng):
    """Each op as a closure over fixed inputs and weights; returns its output tensor."""
    n = 96
    z, mask, w = triangle_case(n, seed=4, mask_p=0.9, perturbed=True)
    zd = torch.from_numpy(z).to("cuda", torch.bfloat16)
    md = torch.from_numpy(mask).cuda()
    tri_w = torch.from_numpy(pack(w)).cuda()
    att_w = torch.from_numpy(_attention_packed(rng)).cuda()
    s, cm = 40, 64
    msa = torch.from_numpy(rng.standard_normal((s, n, cm)).astype(np.float32)).to("cuda", torch.bfloat16)
    msa_mask = torch.ones(s, n, device="cuda")
    opm_w = torch.from_numpy(np.concatenate([np.ones(cm), np.zeros(cm), rng.standard_normal(cm * 32) / 8, np.zeros(32),
                                             rng.standard_normal(cm * 32) / 8, np.zeros(32),
                                             rng.standard_normal(32 * 32 * 128) / 32, np.zeros(128)])
                             .astype(np.float32)).cuda()
    w1 = (rng.standard_normal((128, 512)) / np.sqrt(128)).astype(np.float32)
    w2 = (rng.standard_normal((512, 128)) / np.sqrt(512)).astype(np.float32)
    (c1, s1), (c2, s2) = oracle.quantize_q8_columns(w1), oracle.quantize_q8_columns(w2)
    tw = {"layerNormScale": torch.ones(128, device="cuda"), "layerNormOffset": torch.zeros(128, device="cuda"),
          "firstWeight": af2cuda.Q8Matrix(torch.from_numpy(c1).cuda(), torch.from_numpy(s1).cuda(), "channel"),
          "firstBias": torch.zeros(512, device="cuda"),
          "secondWeight": af2cuda.Q8Matrix(torch.from_numpy(c2).cuda(), torch.from_numpy(s2).cuda(), "channel"),
          "secondBias": torch.zeros(128, device="cuda")}
    lin_w = torch.from_numpy((rng.standard_normal((128, 200)) / np.sqrt(128)).astype(np.float32)).cuda()
    lin_b = torch.from_numpy(rng.standard_normal(200).astype(np.float32)).cuda()
    x = zd.view(n * n, 128)
    torch.cuda.synchronize()  # the inputs are made on torch's stream; the library runs on its own
    return {
        "triangle": lambda: af2cuda.encode_triangle_multiplication_tensors(
            device, 1, zd, md, tri_w, out=torch.empty(n, n, 128, device="cuda"), residual=False),
        "attention": lambda: af2cuda.encode_triangle_attention_tensors(
            device, "ending", zd, md, att_w, 4, out=torch.empty(n, n, 128, device="cuda"), residual=False),
        "opm": lambda: af2cuda.encode_outer_product_mean_tensors(
            device, msa, msa_mask, opm_w, 32, 128, out=torch.empty(n, n, 128, device="cuda"), residual=False),
        "transition": lambda: af2cuda.encode_transition_tensors(
            device, x, tw, out=torch.empty(n * n, 128, device="cuda"), residual=False),
        "linear": lambda: af2cuda.linear_tensors(device, x, lin_w, lin_b, out=torch.empty(n * n, 200, device="cuda")),
    }, tri_w


def test_cached_weights_give_the_same_bits_and_skip_preparation(device):
    import torch
    ops, _ = _ops(device, torch, np.random.default_rng(0))
    uncached = {}
    for name, op in ops.items():
        uncached[name] = op()
    device.sync()
    before = device.memory_snapshot()["currentBytes"]
    device.set_weight_cache(True)
    try:
        for name, op in ops.items():
            first = op()
            device.sync()
            launches = device.launch_count
            again = op()
            device.sync()
            repeat_launches = device.launch_count - launches
            assert torch.equal(first, uncached[name]), name
            assert torch.equal(again, uncached[name]), name
            assert repeat_launches >= 1, name
        assert device.memory_snapshot()["currentBytes"] > before  # the cache holds the prepared copies
    finally:
        device.set_weight_cache(False)
    assert device.memory_snapshot()["currentBytes"] == before


def test_repeat_calls_launch_fewer_kernels(device):
    import torch
    ops, _ = _ops(device, torch, np.random.default_rng(1))
    device.set_weight_cache(True)
    try:
        for name, op in ops.items():
            op()
            device.sync()
            n0 = device.launch_count
            op()
            device.sync()
            cached = device.launch_count - n0
            device.clear_weight_cache()
            n1 = device.launch_count
            op()
            device.sync()
            fresh = device.launch_count - n1
            assert cached < fresh, (name, cached, fresh)
    finally:
        device.set_weight_cache(False)


def test_clearing_the_cache_takes_changed_weights(device):
    import torch
    ops, tri_w = _ops(device, torch, np.random.default_rng(2))
    device.set_weight_cache(True)
    try:
        a = ops["triangle"]()
        device.sync()
        tri_w.mul_(0.5)  # changed in place: stale until the cache is cleared
        torch.cuda.synchronize()
        device.clear_weight_cache()
        b = ops["triangle"]()
        device.sync()
        device.set_weight_cache(False)
        c = ops["triangle"]()
        device.sync()
        assert not torch.equal(a, b)
        assert torch.equal(b, c)
    finally:
        device.set_weight_cache(False)
