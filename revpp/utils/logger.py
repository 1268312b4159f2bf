"""Loggers and system-information logging (BERT/src/logger.py:7-65, logging_utils.py:9-122)."""
from __future__ import annotations

import logging
import os
import platform
import subprocess
import sys
from pathlib import Path
from typing import Optional

import torch


def build_logger(name: str, path: Optional[Path], console: bool = False, level=logging.INFO) -> logging.Logger:
    logger = logging.getLogger(f"revpp.{name}")
    logger.setLevel(level)
    logger.propagate = False
    for h in list(logger.handlers):
        logger.removeHandler(h)
    fmt = logging.Formatter("%(asctime)s [%(levelname)s] %(message)s")
    if path is not None:
        try:
            Path(path).parent.mkdir(parents=True, exist_ok=True)
            fh = logging.FileHandler(path)
            fh.setFormatter(fmt)
            logger.addHandler(fh)
        except OSError:
            pass
    if console:
        sh = logging.StreamHandler(sys.stdout)
        sh.setFormatter(fmt)
        logger.addHandler(sh)
    return logger


def log_sys_info(logger: logging.Logger) -> None:
    logger.info("python %s | torch %s | cuda %s | platform %s", sys.version.split()[0], torch.__version__,
                torch.version.cuda, platform.platform())
    try:
        import psutil

        vm = psutil.virtual_memory()
        logger.info("cpus %d | host memory %.1f GiB", psutil.cpu_count(), vm.total / 2**30)
    except Exception:  # noqa: BLE001
        pass


def log_node_info(logger: logging.Logger) -> None:
    """GPU topology of the node (``nvidia-smi topo --matrix``), as the reference logs it."""
    try:
        out = subprocess.run(["nvidia-smi", "topo", "--matrix"], capture_output=True, text=True, timeout=20)
        if out.returncode == 0:
            logger.info("topology:\n%s", out.stdout)
    except (OSError, subprocess.SubprocessError):
        logger.info("nvidia-smi not available")


def log_gpu_static_info(logger: logging.Logger, device: torch.device) -> None:
    if device.type != "cuda":
        logger.info("device: cpu")
        return
    p = torch.cuda.get_device_properties(device)
    logger.info("device %s: %s, %d SMs, %.1f GiB, cc %d.%d", device, p.name, p.multi_processor_count,
                p.total_memory / 2**30, p.major, p.minor)


def log_model_info(logger: logging.Logger, model: torch.nn.Module) -> None:
    n = sum(p.numel() for p in model.parameters())
    logger.info("stage parameters: %d (%.2f M)", n, n / 1e6)


def log_exp_config(logger: logging.Logger, cfg) -> None:
    for k, v in sorted(vars(cfg).items()):
        logger.info("cfg %s = %s", k, v)
