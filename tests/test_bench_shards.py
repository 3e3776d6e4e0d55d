"""The bench's multi-GPU split on the CPU: for every op, the ranks' shards of one seeded job,
computed independently and stacked the way ``ntilang_b200.dist.gather_rows`` assembles them, give
the whole job's result; and the per-rank work adds up to the whole job's algorithmic work.  The
kernels are stood in for by torch CPU functions of the same op (the GPU path is checked
bit-for-bit against a one-GPU run inside ``bench.py`` itself)."""

from __future__ import annotations

import math

import pytest

import bench

torch = pytest.importorskip("torch")


def small(cls, **sizes):
    return type(f"Small{cls.__name__}", (cls,), dict(sizes))


CASES = {
    "cumsum": (small(bench.CumsumOp, full_rows=37, cols=20), lambda x: torch.cumsum(x, 1)),
    "softmax": (small(bench.SoftmaxOp, full_rows=29, cols=16), lambda x: torch.softmax(x, 1)),
    "rmsnorm": (small(bench.RMSNormOp, full_rows=19, cols=12),
                lambda x, w: x * torch.rsqrt((x * x).mean(1, keepdim=True) + 1e-6) * w),
    "layernorm": (small(bench.LayerNormOp, full_rows=23, cols=8),
                  lambda x, w, b: torch.nn.functional.layer_norm(x, (8,), w, b, 1e-5)),
    "vadd": (small(bench.VaddOp, full_rows=1001), lambda a, b: a + b),
    "pointwise": (small(bench.GenericFmaOp, full_rows=999), lambda a, b, c: a * b + c),
    "transpose": (small(bench.TransposeOp, full_rows=13, cols=7), lambda a: a.t().contiguous()),
    "gemm": (small(bench.GemmOp, m=40, n=24, k=16), lambda a, b: a.float() @ b.float()),
    "gemm_bias_relu": (small(bench.GemmBiasReluOp, m=33, n=8, k=16),
                       lambda a, b, bias: torch.relu(a.float() @ b.float() + bias)),
    "fa2": (small(bench.FA2Op, B=8, H=3, S=16, D=8),
            lambda q, k, v: torch.nn.functional.scaled_dot_product_attention(q.float(), k.float(), v.float())),
    "fa2_causal": (small(bench.FA2CausalOp, B=6, H=2, S=16, D=8),
                   lambda q, k, v: torch.nn.functional.scaled_dot_product_attention(
                       q.float(), k.float(), v.float(), is_causal=True)),
}


def test_every_bench_op_has_a_case():
    assert set(CASES) == set(bench.OPS)


@pytest.mark.parametrize("world", [1, 2, 3, 8])
@pytest.mark.parametrize("name", sorted(CASES))
def test_shards_reassemble_the_whole_job(name, world):
    cls, fn = CASES[name]
    whole = cls(torch, "cpu", 0, 1)
    expect = fn(*whole.global_inputs())
    parts = []
    for rank in range(world):
        op = cls(torch, "cpu", rank, world)
        local = op.slice_inputs(op.global_inputs())
        parts.append(op.gather_view(fn(*local)))
    got = cls(torch, "cpu", 0, world).ungather(torch.cat(parts, 0))
    assert got.shape == expect.shape
    assert torch.equal(got, expect) if name not in ("fa2", "fa2_causal") else torch.allclose(got, expect, atol=1e-5)


@pytest.mark.parametrize("world", [1, 2, 4, 8])
@pytest.mark.parametrize("name", sorted(bench.OPS))
def test_rank_work_adds_up_to_the_baseline_job(name, world):
    """At the BASELINE sizes, the ranks' algorithmic work sums to the whole job (plus, for the
    normalisations, the weight vectors every rank reads)."""
    cls = bench.OPS[name]
    ops = [cls(None, None, r, world) for r in range(world)]
    total = ops[0].total_units()
    assert sum(o.units() for o in ops) == total
    whole = cls(None, None, 0, 1).units()
    extra = {"rmsnorm": 1, "layernorm": 2}.get(name, 0) * ops[0].cols * 4 * (world - 1)
    assert total == whole + extra
    assert max(o.rows for o in ops) - min(o.rows for o in ops) <= 1
    assert math.isclose(sum(o.rows for o in ops), ops[0].full_rows)


@pytest.mark.parametrize("name", sorted(bench.OPS))
def test_weak_leg_runs_the_whole_job_on_every_rank(name):
    """``--gpus N`` also times a full-size job on each rank: that op is the whole job whatever the
    rank's index."""
    whole = bench.whole_job_op(bench.OPS[name], None, None)
    assert whole.world == 1 and whole.rank == 0 and whole.rows == whole.full_rows
    assert whole.total_units() == bench.OPS[name](None, None, 0, 1).units()


@pytest.mark.parametrize("world", [1, 8])
def test_the_json_line_fits_the_driver_tail(world, monkeypatch):
    """The driver keeps the last ~3,000 characters of the bench's stdout: the one-line record, with
    every op's figures at their longest, stays under 2,900."""
    monkeypatch.setattr(bench, "cpu_model", lambda: "Intel(R) Xeon(R) Platinum 8480C Processor @ 2.00GHz x")
    results = {}
    for name in bench.OPS:
        r = {"value": 12345.678, "unit": "GB/s", "ms_per_step": 1.922682, "gpu_launches": 50,
             "roofline": {"bound": "hbm", "achieved": 12345.678, "peak": 6455.6, "unit": "GB/s", "frac": 1.0686,
                          "traffic": 165965158},
             "e2e": {"value": 141.485, "unit": "GB/s", "h2d_bytes_per_step": 201326592,
                     "d2h_bytes_per_step": 67108864}}
        if world == 1:
            r["cpu_baseline"] = {"value": 434.6357, "unit": "GB/s", "cores": 224, "kind": "port",
                                 "sample": "6480 x cumsum [32768,256]"}
            r["cpu_torch"] = {"value": 434.6357, "cores": 224}
        else:
            r["weak"] = {"value": 98765.432, "ms_per_step": 1.922682, "gpu_launches": 50}
            r["verify"] = {"bit_identical": True}
        results[name] = r
    clocks = {"sm_mhz": 1965.0, "sm_max_mhz": 1965.0, "reasons": ["sw_power_cap", "sw_thermal_slowdown"],
              "samples": 1335, "power_w_max": 1000.61}
    line = bench.assemble_line(50, 5, world, results, clocks, f"gpurun_out/bench_detail_n{world}.json")
    text = bench.json.dumps(line)
    assert len(text) <= 2900, len(text)
    assert set(line["ops"]) == set(bench.OPS) and line["n_gpus"] == world and line["value"] == 12345.678
