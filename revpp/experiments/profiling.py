"""Profiling experiment (BERT/experiment/profiling/main.py:19-249).

Runs up to 12 training steps under torch.profiler (CPU + CUDA activity, shapes, memory,
stacks) with the reference's wait / warmup / active = 4 / 4 / 4 schedule (shrunk when
there are fewer batches), and additionally times every step on the device with CUDA
events.  Outputs under ``profiles/{exp_id}/{mbs}x{nmb}/{env_id}/rank{r}/``:

  trace.json                 Chrome trace
  memory.json                memory timeline (torch.profiler export), when available
  performance_stats.json     step times (device, max over ranks), throughput
                             (global batch * active steps / active duration), span stats
  timeline_peak_stats.json   peak allocated / reserved memory, the peak's breakdown by
                             category (torch's memory-timeline categories, as the reference
                             reports them, and this framework's own buffer accounting),
                             and the predicted peak
"""
from __future__ import annotations

import json
import statistics

import torch
import torch.distributed as dist

from revpp.utils.profiling import DeviceTimer, max_over_ranks

from .base import Experiment
from .events import parse_event_spans, span_stats
from .memory_predictor import predict_peak_bytes
from .memory_report import framework_breakdown, profiler_peak_breakdown


class ProfilingExperiment(Experiment):
    batch_limit = 12

    def _sched(self, n: int):
        wait, warm, active = 4, 4, 4
        while wait + warm + active > n and (wait > 0 or warm > 1):
            if wait > 0:
                wait -= 1
            elif warm > 1:
                warm -= 1
        active = max(1, min(active, n - wait - warm))
        return wait, warm, active

    def run(self) -> None:
        cfg, env, t = self.cfg, self.env, self.trainer
        n = min(self.batch_limit, self.loaders.num_batches_train)
        wait, warm, active = self._sched(n)
        out = (cfg.profile_rdir / cfg.exp_id / f"{cfg.microbatch_size}x{cfg.num_microbatches}" / cfg.env_id /
               f"rank{env.rank}")
        out.mkdir(parents=True, exist_ok=True)
        acts = [torch.profiler.ProfilerActivity.CPU]
        if env.device.type == "cuda":
            acts.append(torch.profiler.ProfilerActivity.CUDA)
        timer = DeviceTimer(env.device)
        step_ms = []
        prof = torch.profiler.profile(activities=acts, record_shapes=True, profile_memory=True, with_stack=True,
                                      schedule=torch.profiler.schedule(wait=wait, warmup=warm, active=active))
        loader = iter(self.loaders.train_loader) if t.is_first else None
        if env.device.type == "cuda":
            torch.cuda.reset_peak_memory_stats()
        with prof:
            for i in range(n):
                batch = next(loader) if loader is not None else None
                timer.start()
                t.train_step(batch)
                step_ms.append(timer.stop())
                prof.step()
        prof.export_chrome_trace(str(out / "trace.json"))
        try:
            if env.device.type == "cuda":
                prof.export_memory_timeline(str(out / "memory.json"), device=str(env.device))
        except Exception:  # noqa: BLE001  (memory timeline needs the memory profile; optional)
            pass
        active_ms = step_ms[-active:]
        local = statistics.mean(active_ms)
        step_max = max_over_ranks(local, env.device)
        spans = parse_event_spans(out / "trace.json")
        stats = {
            "avg_step_time_ms_local": local,
            "avg_step_time_ms": step_max,
            "throughput_samples_per_sec": cfg.batch_size / (step_max / 1e3),
            "step_times_ms": step_ms,
            "active_steps": active,
            "schedule": {"wait": wait, "warmup": warm, "active": active},
            "spans": span_stats(spans),
            "world_size": env.world_size,
            "microbatch_size": cfg.microbatch_size,
            "num_microbatches": cfg.num_microbatches,
        }
        (out / "performance_stats.json").write_text(json.dumps(stats, indent=2))
        peak = {}
        if env.device.type == "cuda":
            alloc = torch.cuda.max_memory_allocated()
            peak = {"cuda_max_alloc_gib": alloc / 2**30,
                    "cuda_max_reserved_gib": torch.cuda.max_memory_reserved() / 2**30,
                    "framework_peak_breakdown_gib": framework_breakdown(t, alloc)}
            prof_peak = profiler_peak_breakdown(out / "memory.json")
            if prof_peak is not None:
                peak.update(prof_peak)
        peak["predicted_peak_gib"] = predict_peak_bytes(cfg, t.stage_index, t.P, t.stage.kind,
                                                        pareprop=cfg.is_pareprop) / 2**30
        (out / "timeline_peak_stats.json").write_text(json.dumps(peak, indent=2))
        if env.main_logger:
            env.main_logger.info("profiling: %.2f ms/step (max over ranks), %.1f samples/s, peak %s",
                                 step_max, stats["throughput_samples_per_sec"], peak)
