"""CLI / config invariants, experiment ids, the checkpoint layout, the memory predictor and
the three experiments end to end, all on CPU (gloo for the multi-rank runs)."""
import os
import socket
import subprocess
import sys

import pytest
import torch

from revpp.config import build_global_config, make_exp_id, parse_args
from revpp.experiments.memory_predictor import max_microbatch_for_budget, predict_breakdown

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _cfg(argv: str):
    return build_global_config(parse_args(argv.split()))


# ------------------------------------------------------------------ config / CLI
def test_exp_id_matches_reference_format():
    # BERT/src/config.py:86-105: note the missing separator after "inverse"
    assert make_exp_id("training", "pp", True, True, False, False, "torch.bfloat16", "imdb", 0, 24) == \
        "training_pp_pareprop_torch.bfloat16_imdb_seed0000numLayer24"
    assert make_exp_id("profiling", "pp", True, False, True, False, "torch.float32", "imdb", 3, 12) == \
        "profiling_pp_inversetorch.float32_imdb_seed0003numLayer12"
    assert make_exp_id("training", "none", False, False, False, True, "torch.float32", "cifar10", 7, 4) == \
        "training_none_wcp_torch.float32_cifar10_seed0007numLayer4"
    assert make_exp_id("training", "ddp", False, False, False, False, "torch.float16", "imdb", 0, 2).startswith(
        "training_ddp_std_")


def test_config_invariants():
    base = "--preset tiny-bert --device cpu --dataset synthetic "
    with pytest.raises(Exception):
        _cfg(base + "--batch-size 16 --microbatch-size 4 --num-microbatches 3")
    with pytest.raises(Exception):
        _cfg(base + "--batch-size 16 --microbatch-size 4 --num-microbatches 4 --is_pareprop")
    with pytest.raises(Exception):
        _cfg(base + "--batch-size 16 --microbatch-size 4 --num-microbatches 4 --inverse")
    cfg = _cfg(base + "--batch-size 16 --microbatch-size 4 --num-microbatches 4 --reversible --is_pareprop "
                      "--par-mode pp --autocast-dtype bf16")
    assert cfg.reversible and cfg.is_pareprop and cfg.autocast_dtype == torch.bfloat16
    # the id carries the CLI spelling of the dtype (BERT/src/config.py:102), the checkpoint
    # directory str(torch.dtype) (BERT/src/ckpt_io.py:17)
    assert cfg.exp_id == "training_pp_pareprop_bf16_synthetic_seed0000numLayer4"


# ------------------------------------------------------------------ memory predictor
def test_reversible_activation_memory_is_constant_in_depth_and_layers():
    cfg = _cfg("--preset bert-large --device cpu --batch-size 512 --microbatch-size 16 --num-microbatches 32 "
               "--reversible --par-mode pp --autocast-dtype bf16")
    # a middle stage: same activation bytes at any depth and any number of blocks per stage
    acts = [predict_breakdown(cfg, 1, P, "reversible")["activations"] for P in (3, 4, 8)]
    assert acts[0] == acts[1] == acts[2]
    deep = cfg.with_(num_hidden_layers=48)
    assert predict_breakdown(deep, 1, 4, "reversible")["activations"] == acts[1]
    # standard stages keep every block of every in-flight micro-batch: grows with depth
    assert predict_breakdown(deep, 0, 4, "standard")["activations"] > \
        predict_breakdown(cfg, 0, 4, "standard")["activations"]


def test_paber_microbatch_fits_budget_and_grows_with_it():
    cfg = _cfg("--preset bert-large --device cpu --batch-size 512 --microbatch-size 16 --num-microbatches 32 "
               "--reversible --par-mode pp --autocast-dtype bf16")
    small = max_microbatch_for_budget(cfg, 4, "reversible", 20 << 30)
    large = max_microbatch_for_budget(cfg, 4, "reversible", 160 << 30)
    assert 1 <= small < large


# ------------------------------------------------------------------ checkpoint layout
def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def test_checkpoint_round_trip_with_reference_alias_keys(tmp_path):
    from revpp.ckpt import ckpt_dir, file_name, load_checkpoint, save_checkpoint
    from revpp.data import SyntheticBatches
    from revpp.engine import Trainer
    from revpp.utils.env import build_env

    cfg = _cfg(f"--preset tiny-bert --num-hidden-layers 2 --device cpu --batch-size 8 --microbatch-size 4 "
               f"--num-microbatches 2 --reversible --lr 1e-3 --checkpoint-dir {tmp_path} --log-dir {tmp_path}/logs")
    env = build_env(cfg)
    tr = Trainer(cfg, env)
    batch = SyntheticBatches(cfg, 8, 1, seed=1).make(0)
    tr.train_step(batch)
    path = save_checkpoint(tr, cfg, 0, epoch=3)
    assert path == ckpt_dir(cfg) / file_name(cfg, 0) and path.name == "latest.pth"
    sd = torch.load(path)
    plain = [k for k in sd if ".layers.0.F." in k]
    aliased = [k for k in sd if ".layers.0.block.F." in k]
    assert plain and len(plain) == len(aliased)
    saved = {k: v.clone() for k, v in tr.module.state_dict().items()}
    m_saved = tr.flat.exp_avg.clone()
    with torch.no_grad():
        tr.flat.data.add_(1.0)
        tr.flat.exp_avg.zero_()
    st = load_checkpoint(tr, cfg, 0)
    assert st is not None and st["epoch"] == 3
    for k, v in tr.module.state_dict().items():
        assert torch.equal(v, saved[k]), k
    assert torch.equal(tr.flat.exp_avg, m_saved)
    # a file with only the aliased spelling (as the reference writes it for wrapped blocks)
    only_alias = {k: v for k, v in sd.items() if ".layers." not in k or ".block." in k}
    torch.save(only_alias, path)
    with torch.no_grad():
        tr.flat.data.zero_()
    load_checkpoint(tr, cfg, 0)
    for k, v in tr.module.state_dict().items():
        assert torch.equal(v, saved[k]), k


# ------------------------------------------------------------------ experiments through main.py
def _main(tmp_path, extra: str, world: int = 2):
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={world}",
           "--master-addr=127.0.0.1", f"--master-port={_port()}", os.path.join(ROOT, "main.py")]
    cmd += (f"--preset tiny-bert --num-hidden-layers 4 --device cpu --dataset synthetic --synthetic-batches 2 "
            f"--batch-size 16 --microbatch-size 4 --num-microbatches 4 --par-mode pp --reversible --lr 1e-3 "
            f"--num-epochs 1 --log-dir {tmp_path}/logs --checkpoint-dir {tmp_path}/ckpt "
            f"--profile-dir {tmp_path}/prof " + extra).split()
    env = dict(os.environ, OMP_NUM_THREADS="1")
    p = subprocess.run(cmd, capture_output=True, text=True, timeout=600, cwd=ROOT, env=env)
    assert p.returncode == 0, p.stdout[-3000:] + p.stderr[-3000:]
    return p


def test_training_experiment_cli(tmp_path):
    _main(tmp_path, "-e training --save-checkpoint")
    assert list((tmp_path / "logs").rglob("metrics.csv")), list((tmp_path / "logs").rglob("*"))
    assert sorted(p.name for p in (tmp_path / "ckpt").rglob("latest_rank*.pth")) == \
        ["latest_rank0.optim.pth", "latest_rank0.pth", "latest_rank1.optim.pth", "latest_rank1.pth"]


def test_actv_err_experiment_cli(tmp_path):
    _main(tmp_path, "-e actv-err")
    files = list(tmp_path.rglob("*.csv"))
    assert files, list(tmp_path.rglob("*"))


def test_profiling_experiment_cli(tmp_path):
    _main(tmp_path, "-e profiling")
    stats = list((tmp_path / "prof").rglob("performance_stats.json"))
    assert len(stats) == 2, list((tmp_path / "prof").rglob("*"))


def test_bench_paber_microbatch_default(monkeypatch):
    """bench.py picks the expanded micro-batch on a single stage and 16 with a pipeline,
    and an explicit --microbatch-size wins."""
    import importlib.util
    import sys

    spec = importlib.util.spec_from_file_location("bench_mod", os.path.join(ROOT, "bench.py"))
    bench = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(bench)
    for argv, want in ((["--gpus", "1"], 64), (["--gpus", "2"], 16), (["--gpus", "8"], 16),
                       (["--gpus", "2", "--dp", "2"], 64), (["--gpus", "1", "--microbatch-size", "32"], 32)):
        monkeypatch.setattr(sys, "argv", ["bench.py"] + argv)
        a = bench.parse()
        assert a.microbatch_size == want, (argv, a.microbatch_size)
        assert a.global_batch % (a.microbatch_size * a.dp) == 0


def test_profiler_peak_breakdown_from_memory_timeline(tmp_path):
    """The peak of a memory timeline export and its split by category, as the reference's
    timeline_peak_stats.json reports it."""
    import json

    from revpp.experiments.memory_report import BASE_CATS, profiler_peak_breakdown

    G = 1 << 30
    rows = [[0] * len(BASE_CATS) for _ in range(3)]
    rows[1][BASE_CATS.index("PARAMETER")] = 2 * G
    rows[1][BASE_CATS.index("ACTIVATION")] = 3 * G
    rows[2][BASE_CATS.index("PARAMETER")] = 2 * G
    rows[2][BASE_CATS.index("CATEGORY_0")] = 9 * G  # not a plotted category
    path = tmp_path / "memory.json"
    path.write_text(json.dumps([[1000, 2000, 3000], rows]))
    r = profiler_peak_breakdown(path)
    assert r["peak_total_gib"] == 5.0 and r["timestamp_ms"] == 1.0
    assert r["profiler_peak_breakdown_gib"] == {"PARAMETER": 2.0, "ACTIVATION": 3.0}
    assert profiler_peak_breakdown(tmp_path / "missing.json") is None


@pytest.mark.parametrize("script", ["bert_actv_err.sh", "vit_profiling.sh"])
def test_launch_scripts_run_small(tmp_path, script):
    """The launch scripts of the reference's run configurations start the CLI with its
    flags; later flags (EXTRA) shrink the model so the run fits a CPU test."""
    extra = (f"--device cpu --synthetic-batches 1 --num-hidden-layers 4 --hidden-size 64 --num-attention-heads 2 "
             f"--batch-size 8 --microbatch-size 2 --num-microbatches 4 --log-dir {tmp_path}/logs "
             f"--profile-dir {tmp_path}/prof --checkpoint-dir {tmp_path}/ckpt")
    if script.startswith("bert"):
        extra += " --max-position-embeddings 32"
    else:
        extra += " --img-size 32 --patch-size 16"
    env = dict(os.environ, NPROC="2", DATASET="synthetic", DTYPE="fp32", EXTRA=extra, MASTER_PORT=str(_port()),
               OMP_NUM_THREADS="1")
    p = subprocess.run(["bash", os.path.join(ROOT, "launch", script)], capture_output=True, text=True, timeout=600,
                       cwd=ROOT, env=env)
    assert p.returncode == 0, p.stdout[-2000:] + p.stderr[-2000:]


def test_bench_pipeline_defaults(monkeypatch):
    """With a pipeline, this framework's arm uses copy-engine channels and interleaved 1F1B with
    as many chunks per rank as the blocks allow (at most 3); NCCL groups and the reference arm
    keep plain 1F1B."""
    import importlib.util
    import sys

    spec = importlib.util.spec_from_file_location("bench_mod2", os.path.join(ROOT, "bench.py"))
    bench = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(bench)
    cases = ((["--gpus", "1"], "1f1b", 1), (["--gpus", "2"], "interleaved", 3), (["--gpus", "8"], "interleaved", 3),
             (["--gpus", "4", "--p2p", "group"], "1f1b", 1), (["--gpus", "8", "--impl", "reference"], "1f1b", 1))
    for argv, sched, v in cases:
        monkeypatch.setattr(sys, "argv", ["bench.py"] + argv)
        a = bench.parse()
        assert a.schedule == sched and a.virtual_stages == v, (argv, a.schedule, a.virtual_stages)
        if "--p2p" not in argv:
            assert a.p2p == "copy"
