"""Multi-GPU placement host logic on CPU: world_size-2 gloo groups.

Each rank plays one GPU's client group (HP + BE threads running CPU stand-in
steps, no interposer), the results are gathered on rank 0 over gloo and
aggregated the way kernel_intercept_b200.launch reports them.
"""
import json
import os
import socket
import time

import pytest
import torch.multiprocessing as mp

from kernel_intercept_b200 import launch


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_body(rank, world, port, out_dir):
    import datetime

    import torch.distributed as dist
    os.environ.update({"MASTER_ADDR": "127.0.0.1", "MASTER_PORT": str(port)})
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    gpu = launch.placement(rank, world, visible=world)
    hp_ms = 2.0 + rank  # rank 1's HP is slower: the aggregate p99 must see it

    def hp():
        time.sleep(hp_ms / 1e3)

    def be():
        time.sleep(0.001)

    res = launch.run_group([(hp, 1), (be, 256)], num_iters=20)
    res["rank"] = rank
    res["gpu"] = gpu
    groups = launch.gather(res, rank, world)
    dist.destroy_process_group()
    if rank == 0:
        with open(os.path.join(out_dir, "report.json"), "w") as f:
            json.dump({"report": launch.report(groups), "groups_full": groups}, f)


def test_two_groups_gather_and_aggregate(tmp_path):
    port = _port()
    mp.spawn(_rank_body, args=(2, port, str(tmp_path)), nprocs=2, join=True)
    data = json.load(open(tmp_path / "report.json"))
    rep = data["report"]
    agg = rep["aggregate"]
    assert agg["groups"] == 2 and agg["errors"] == []
    assert sorted(g["gpu"] for g in rep["groups"]) == [0, 1]
    for g in rep["groups"]:
        assert [c["client_type"] for c in g["clients"]] == ["HP", "BE"]
        assert g["clients"][0]["num_iters"] == 20
        assert "latencies_ms" not in g["clients"][0]
    # p99 over both groups' HP iterations is at least rank 1's sleep (3 ms)
    lat = [x for g in data["groups_full"] for x in g["clients"][0]["latencies_ms"]]
    assert len(lat) == 40
    assert agg["hp_p99_ms"] == pytest.approx(launch.percentile(lat, 0.99))
    assert agg["hp_p99_ms"] >= 3.0
    # BE throughput is the sum of both groups
    be = sum(g["clients"][1]["units_per_s"] for g in data["groups_full"])
    assert agg["be_units_per_s"] == pytest.approx(be)


def test_placement_one_group_per_gpu():
    assert [launch.placement(r, 4, 8) for r in range(4)] == [0, 1, 2, 3]
    with pytest.raises(ValueError):
        launch.placement(0, 9, 8)


def test_aggregate_reports_client_errors():
    groups = [{"rank": 0, "clients": [
        {"client_idx": 0, "latencies_ms": [1.0, 2.0], "units_per_s": 10.0},
        {"client_idx": 1, "error": "RuntimeError('boom')"}]}]
    agg = launch.aggregate(groups)
    assert agg["errors"] == [(0, 1, "RuntimeError('boom')")]
    assert agg["hp_units_per_s"] == 10.0 and agg["be_units_per_s"] == 0.0


def test_bench_reference_arm_other_ranks_exit_quietly(capsys):
    """Under torchrun the reference arm runs on rank 0 only."""
    import bench
    os.environ["RANK"] = "1"
    try:
        assert bench.run_reference(type("A", (), {"steps": 1, "warmup": 0, "gpus": 2})()) == 0
    finally:
        os.environ.pop("RANK")
    assert capsys.readouterr().out == ""


def test_bench_roofline_is_the_hp_clients_dominant_op():
    """The roofline's op class, rate and share come from the HP client's
    timed ops alone: a BE op's events also span the time it spends stopped."""
    import bench
    recs = [{"client": 0, "op_type": "CUBLAS_GEMM_EX", "duration_ms": 0.5, "work": 1e12,
             "kernel_id": "kx_gemm_tc<bn256,bf16,Ak,Bk>"} for _ in range(4)]
    recs += [{"client": 0, "op_type": "CUBLAS_SGEMM", "duration_ms": 1.0, "work": 1e10,
              "kernel_id": "kx_gemm_tc<bn64,f32x3,Ak,Bk>"}]
    recs += [{"client": 1, "op_type": "CUDNN_CONV_FWD", "duration_ms": 500.0, "work": 1e12,
              "kernel_id": "kx_conv_fwd_tc<bn128,f32x3,im2col>"}]
    r = bench.roofline(recs, {"bf16_tflops": 1600.0, "bf16_tflops_sustained": 1400.0},
                       "test", 700.0, True, 4)
    assert r["op"] == "HP:CUBLAS_GEMM_EX" and r["launches_timed"] == 4
    assert r["achieved"] == pytest.approx(2000.0)  # 1e12 FLOP in 0.5 ms
    assert r["peak"] == 1400.0 and r["frac"] == pytest.approx(2000.0 / 1400.0, rel=1e-3)
    assert r["share_of_hp_captured_ms"] == pytest.approx(2.0 / 3.0, rel=1e-3)
    assert "fp32_3xtf32_ceiling" not in r
