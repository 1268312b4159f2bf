"""Experiment assembly (BERT/experiment/base.py:57-317): seeding, logging, data, trainer,
engine, checkpoint load / save.  Subclasses implement ``run``."""
from __future__ import annotations

import time
from abc import ABC, abstractmethod
from typing import Optional

from revpp.ckpt import load_checkpoint, save_checkpoint
from revpp.config import GlobalConfig
from revpp.data import LoaderBundle, build_loaders
from revpp.engine import Engine, Trainer
from revpp.metrics import MetricTracker
from revpp.utils.env import EnvContext
from revpp.utils.logger import log_exp_config, log_gpu_static_info, log_model_info, log_node_info, log_sys_info
from revpp.utils.seed import set_seed


class Experiment(ABC):
    eval_actv_err = False

    def __init__(self, cfg: GlobalConfig, env: EnvContext):
        self.cfg = cfg
        self.env = env
        self.trainer: Optional[Trainer] = None
        self.engine: Optional[Engine] = None
        self.loaders: Optional[LoaderBundle] = None
        self.t0 = time.time()
        self.start_epoch = 0
        set_seed(cfg.seed + env.rank, deterministic=True)
        if env.main_logger:
            log_sys_info(env.main_logger)
            log_exp_config(env.main_logger, cfg)
        if env.node_logger:
            log_node_info(env.node_logger)
        env.proc_logger.info("global rank %d, local rank %d", env.rank, env.local_rank)
        log_gpu_static_info(env.proc_logger, env.device)

    def before_run(self) -> None:
        cfg, env = self.cfg, self.env
        self.trainer = Trainer(cfg, env, eval_actv_err=self.eval_actv_err)
        t = self.trainer
        if env.main_logger:
            log_model_info(env.main_logger, t.module)
        self.loaders = build_loaders(cfg, env.rank, env.world_size, t.P, env.device, loads_data=t.is_first)
        if cfg.load_checkpoint:
            st = load_checkpoint(t, cfg, env.rank)
            if st is not None:
                self.start_epoch = int(st.get("epoch", 0))
        log_dir = cfg.log_rdir / cfg.exp_id / cfg.env_id
        tracker = MetricTracker(cfg.num_classes, (1, 5), cfg.num_epochs, env.device, env.main_logger,
                                csv_path=log_dir / "metrics.csv")
        self.engine = Engine(t, self.loaders, tracker)

    @abstractmethod
    def run(self) -> None:
        ...

    def after_run(self) -> None:
        if self.cfg.save_checkpoint and self.trainer is not None:
            save_checkpoint(self.trainer, self.cfg, self.env.rank, epoch=self.start_epoch + self.cfg.num_epochs)
        if self.trainer is not None:
            self.trainer.close()
        if self.env.main_logger:
            self.env.main_logger.info("===== experiment complete (%.1f s) =====", time.time() - self.t0)
        self.env.close()
