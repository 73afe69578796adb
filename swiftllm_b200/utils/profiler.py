"""Step profiler: ``SWIFTLLM_PROFILE=<dir>`` records a window of engine
steps with torch.profiler (CPU ops, and CUDA kernels when a GPU is present)
and writes a Chrome trace plus a per-op summary table into <dir>.

  SWIFTLLM_PROFILE=/tmp/prof          output directory ("1": ./swiftllm_profile)
  SWIFTLLM_PROFILE_SKIP=5             steps run before recording starts
  SWIFTLLM_PROFILE_STEPS=20           steps recorded

Files: ``trace.json`` (chrome://tracing / Perfetto) and ``summary.txt``
(ops sorted by device time, or CPU time without a GPU). Off (one integer
compare per step) when the variable is unset. Kernel timings taken under
the profiler are for reading shares, not for reporting.

Parity: the reference's tracing is log-level driven (RUST_LOG / tracing
spans, crates/swiftllm-server/src/main.rs:37-60); this adds the kernel
timeline that a GPU engine needs.
"""

from __future__ import annotations

import os
from typing import Optional

from .logging import get_logger

log = get_logger(__name__)


class StepProfiler:
    def __init__(self, out_dir: Optional[str] = None, skip: Optional[int] = None,
                 steps: Optional[int] = None):
        env = os.environ.get("SWIFTLLM_PROFILE", "")
        out_dir = out_dir if out_dir is not None else ("swiftllm_profile" if env == "1" else env)
        self.out_dir = out_dir or None
        self.skip = int(os.environ.get("SWIFTLLM_PROFILE_SKIP", "5")) if skip is None else skip
        self.steps = int(os.environ.get("SWIFTLLM_PROFILE_STEPS", "20")) if steps is None else steps
        self.n = 0
        self.prof = None
        self.done = self.out_dir is None

    def step(self) -> None:
        """Call once after every engine step."""
        if self.done:
            return
        self.n += 1
        if self.prof is None and self.n == self.skip:
            self._start()
        elif self.prof is not None and self.n >= self.skip + self.steps:
            self._stop()

    def _start(self) -> None:
        import torch
        acts = [torch.profiler.ProfilerActivity.CPU]
        if torch.cuda.is_available():
            acts.append(torch.profiler.ProfilerActivity.CUDA)
        self.prof = torch.profiler.profile(activities=acts, record_shapes=False)
        self.prof.__enter__()
        log.info("profiling steps %d..%d into %s", self.n + 1, self.n + self.steps, self.out_dir)

    def _stop(self) -> None:
        import torch
        if torch.cuda.is_available():
            torch.cuda.synchronize()
        self.prof.__exit__(None, None, None)
        os.makedirs(self.out_dir, exist_ok=True)
        self.prof.export_chrome_trace(os.path.join(self.out_dir, "trace.json"))
        key = "self_cuda_time_total" if torch.cuda.is_available() else "self_cpu_time_total"
        with open(os.path.join(self.out_dir, "summary.txt"), "w") as f:
            f.write(self.prof.key_averages().table(sort_by=key, row_limit=60))
        log.info("profile written to %s", self.out_dir)
        self.prof = None
        self.done = True

    def close(self) -> None:
        """Write what was recorded if the engine stops inside the window."""
        if self.prof is not None:
            self._stop()
