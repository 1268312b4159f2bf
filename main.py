"""revpp command line: one entry point for reversible BERT and ViT pipeline training.

    torchrun --nproc-per-node 4 --master-addr 127.0.0.1 main.py --par-mode pp --reversible \
        --preset bert-large --autocast-dtype bf16 --batch-size 512 --microbatch-size 16 \
        --num-microbatches 32 -e profiling

Same flags as the reference's BERT/main.py and Vit/main.py (plus --model / --preset / --dp /
--schedule / --dataset synthetic); see revpp/config.py.
"""
from __future__ import annotations

import multiprocessing as mp
import sys

from revpp.config import ExpMode, build_global_config, parse_args
from revpp.experiments import EXP_REGISTRY
from revpp.utils.env import build_env


def main(argv=None) -> int:
    args = parse_args(argv)
    cfg = build_global_config(args)
    if cfg.exp_mode == ExpMode.ACC:
        raise SystemExit("--exp-mode acc has no implementation (the reference registers none either)")
    env = build_env(cfg)
    exp = EXP_REGISTRY[cfg.exp_mode.value](cfg, env)
    exp.before_run()
    exp.run()
    exp.after_run()
    return 0


if __name__ == "__main__":
    try:
        mp.set_start_method("fork")
    except RuntimeError:
        pass
    sys.exit(main())
