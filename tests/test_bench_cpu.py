"""CPU checks of the benchmark's FLOP accounting: the kernel-cost.ts formulas
(src/runtime/kernel-cost.ts:71,106-108,148-149,158-162) evaluated at the
BASELINE configs give the per-config figures the throughput is quoted on."""
import sys
from pathlib import Path

import pytest

sys.path.insert(0, str(Path(__file__).resolve().parent.parent))
import bench  # noqa: E402


@pytest.mark.parametrize("gflop,value", [
    (3.758, lambda: bench.triangle_flops(128)),                                     # config 1
    (17.18, lambda: 4.0 * 65536 * 128 * 512),                                       # config 2
    (90.19, lambda: bench.opm_flops(256, 512)),                                     # config 3
    (1404.5, lambda: bench.block_flops(768, 512)),                                  # config 4
    (7146.8, lambda: 2 * bench.triangle_flops(2048) + bench.transition_flops(2048)),  # config 5
    (2628.52, lambda: bench.block_flops()),                                         # the metric's block (962.1 + 1391.6 + 274.9)
    (481.04, lambda: bench.triangle_flops(1024)),                                   # one direction at N=1024
])
def test_flop_counts_of_the_configs(gflop, value):
    assert value() / 1e9 == pytest.approx(gflop, abs=0.06)


def test_kernel_flops_add_up_to_the_block():
    per_kernel = sum(bench.kernel_step_flops(k) for k in
                     ("triangle.contract", "triangle.project", "triangle.output", "opm.fused", "opm.project",
                      "transition.fused"))
    # the triangle's gate projection is counted inside triangle.output (the z . W_g GEMM)
    assert per_kernel == pytest.approx(bench.block_flops(), rel=1e-12)


def test_sharded_kernel_flops_split_over_ranks():
    for world in (2, 4, 8):
        assert bench.kernel_step_flops("triangle.contract", world) * world == \
            pytest.approx(bench.kernel_step_flops("triangle.contract"))


def test_every_workload_is_described():
    assert set(bench.WORKLOADS) == {"tri128", "transition", "opm", "block768", "multimer", "msa_transition",
                                    "triangle_attention", "pair_block"}


def test_attention_flops_follow_kernel_cost():
    # kernel-cost.ts:79-92 at N=1024, c_z=128, 4 heads of 32: project 137.4 + flash 549.8 + output 34.4
    # + pair bias 1.07 GFLOP per direction
    assert bench.attention_flops(1024) / 1e9 == pytest.approx(722.63, abs=0.01)
    per_kernel = sum(bench.kernel_step_flops(k) for k in ("attention.flash", "attention.project", "attention.output"))
    assert per_kernel == pytest.approx(2 * bench.attention_flops(1024), rel=1e-12)
