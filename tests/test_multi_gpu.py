"""Multi-GPU tests (NCCL, one process per GPU).  Skipped with fewer than 2 GPUs."""
import json
import os
import shutil
import socket
import subprocess
import sys
import tempfile

import pytest
import torch

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _run(mode, n=2, timeout=240, args=""):
    if torch.cuda.device_count() < n:
        pytest.skip(f"needs {n} GPUs")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={n}",
           "--master-addr=127.0.0.1", f"--master-port={_port()}", os.path.join(HERE, "_mgpu_worker.py"), mode]
    res_dir = tempfile.mkdtemp(prefix="revpp_mgpu_")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0", REVPP_MGPU_RESULT_DIR=res_dir, REVPP_MGPU_ARGS=args)
    p = subprocess.run(cmd, capture_output=True, text=True, timeout=timeout, env=env)
    if p.returncode != 0:
        # full worker output for post-mortems when REVPP_TEST_LOG_DIR names an existing folder
        out_dir = os.environ.get("REVPP_TEST_LOG_DIR")
        if out_dir and os.path.isdir(out_dir):
            tag = mode + ("_" + args.replace(",", "_").replace("=", "") if args else "")
            with open(os.path.join(out_dir, f"mgpu_{tag}_fail.log"), "w") as fh:
                fh.write(p.stdout + "\n----- stderr -----\n" + p.stderr)
    assert p.returncode == 0, p.stdout[-3000:] + p.stderr[-3000:]
    res = []
    for name in sorted(os.listdir(res_dir)):
        with open(os.path.join(res_dir, name)) as fh:
            res.append(json.load(fh))
    shutil.rmtree(res_dir, ignore_errors=True)
    assert len(res) == n, p.stdout[-2000:]
    return sorted(res, key=lambda r: r["rank"])


def test_pipeline_two_stages_matches_single_stage():
    res = _run("pipeline")
    r0 = res[0]
    assert abs(r0["pp_loss"] - r0["single_loss"]) < 2e-2 * max(1.0, abs(r0["single_loss"]))
    last = res[-1]["losses"]
    assert all(l == l for l in last)
    assert all(r["status"] == 0 for r in res)


def test_fused_replica_allreduce_matches_nccl():
    res = _run("dp")
    for r in res:
        assert r["fused"] == "FusedP2PReducer"
        assert r["status"] == 0
        assert r["max_diff"] <= 1e-3 * max(r["max_step"], 1e-6) + 1e-7, r
        assert r["replica_diff"] == 0.0


@pytest.mark.parametrize("n,args", [
    (2, "p2p=group"),
    (2, "p2p=copy"),
    (2, "p2p=copy,schedule=interleaved,v=2"),
    (4, "p2p=copy"),
    (4, "p2p=copy,schedule=interleaved,v=2"),
])
def test_pipeline_gradients_match_single_stage(n, args):
    """Every parameter gradient of a pipelined step (kernel path, bf16) matches the same
    weights run as one stage: gradients and reconstructed inputs cross stage boundaries
    correctly, over NCCL groups and over copy-engine channels, with 1F1B and interleaved."""
    res = _run("grads", n=n, args=args)
    r0 = res[0]
    assert r0["missing"] == [], r0["missing"][:5]
    assert abs(r0["pp_loss"] - r0["single_loss"]) < 1e-3 * max(1.0, abs(r0["single_loss"])), r0
    assert r0["worst_rel"] < 2e-2, (r0["worst_name"], r0["worst_rel"])
    assert all(r["status"] == 0 for r in res)
    want = args.split("p2p=")[1].split(",")[0]
    assert all(r["p2p"] == want for r in res)


def test_activation_memory_independent_of_pipeline_depth():
    """Reversible stages: the per-GPU memory a training step allocates on top of the
    persistent state does not grow with pipeline depth (PP = 2 vs PP = 4, 2 blocks each)."""
    if torch.cuda.device_count() < 4:
        pytest.skip("needs 4 GPUs")
    t2 = max(r["transient"] for r in _run("memory", n=2, args="p2p=copy"))
    t4 = max(r["transient"] for r in _run("memory", n=4, args="p2p=copy"))
    assert t4 <= 1.05 * t2 + (16 << 20), (t2, t4)
