"""Host-side pieces of bench.py: the sharded input draws of the large
configuration must be exactly the slices of one sequential draw."""
import numpy as np

import bench


def test_large_draw_is_a_slice_of_the_sequential_draw():
    full = 1.0 + 1e-7 * np.random.default_rng(4).uniform(-1.0, 1.0, (40, 24))
    for r0, r1 in ((0, 7), (7, 23), (23, 40)):
        part = bench.large_draw(r0 * 24, (r1 - r0, 24))
        assert np.array_equal(part, full[r0:r1])


def test_shard_rows_tile_the_range():
    for n, world in ((65536, 8), (4096, 3), (10, 4)):
        parts = [bench.shard_rows(n, r, world) for r in range(world)]
        assert parts[0][0] == 0 and parts[-1][1] == n
        assert all(a[1] == b[0] for a, b in zip(parts, parts[1:]))


def _args(**kw):
    import argparse
    base = dict(gpus=1, steps=1, warmup=3, impl="reference", workload="gemm", algorithm="tensor",
                no_secondary=True, kernels_only=False, n=0)
    base.update(kw)
    return argparse.Namespace(**base)


REQUIRED = {"impl", "metric", "value", "unit", "n_gpus", "steps", "warmup", "higher_is_better",
            "scaling", "vs_baseline", "config", "cpu_baseline", "e2e"}


def test_reference_arm_gemm_line():
    line = bench.run_reference(_args())
    assert REQUIRED <= set(line)
    assert line["impl"] == "reference" and line["value"] > 0
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["e2e"]["value"] == line["value"]
    assert line["metric"] == bench.METRIC
    # the same workload dict as the GPU arm's line, one full 4096^3 per step
    assert line["config"] == bench.gemm_config(1, "tensor")


def test_reference_arm_stream_line():
    line = bench.run_reference_stream(_args(workload="fused_add_mul", n=1 << 20))
    assert REQUIRED <= set(line)
    assert line["cpu_baseline"]["kind"] == "port" and line["value"] > 0


def test_reference_arm_uses_every_host_core_under_torchrun(monkeypatch):
    """torchrun sets OMP_NUM_THREADS=1 in each rank; the CPU arms still run
    numpy's BLAS on every host core and report the count they used."""
    with bench.all_host_threads() as pool:
        assert pool.threads == bench.host_cores()
