"""Metrics callbacks of the reference (scao/logging.py): ``collect_metrics``
and the console / TensorBoard / Weights & Biases sinks, same names, keys and
output format, for ``SCAO.add_callback``.  Host code only; the metrics are
read when a callback is registered (ranks and the int8 factors' absmax are
small device reads)."""
from __future__ import annotations

import math
from typing import Callable

MetricsDict = dict
Callback = Callable[[MetricsDict], None]


def _due(metrics, every):
    step = metrics.get("step", 0)
    return not (isinstance(step, int) and step % every != 0), step


class ConsoleLogger:
    """Print the metrics every ``log_every`` steps as
    ``<prefix> step=S  key=value ...`` (floats with 4 decimals)
    (scao/logging.py:61-86)."""

    def __init__(self, log_every: int = 100, prefix: str = "[SCAO]") -> None:
        self.log_every = log_every
        self.prefix = prefix

    def __call__(self, metrics: MetricsDict) -> None:
        due, step = _due(metrics, self.log_every)
        if not due:
            return
        fields = [f"step={step}"] + [
            f"{k}={v:.4f}" if isinstance(v, float) else f"{k}={v}"
            for k, v in metrics.items() if k != "step"]
        print(self.prefix + " " + "  ".join(fields))


class TensorBoardLogger:
    """``writer.add_scalar`` of every numeric metric (booleans as 0 / 1, NaN
    skipped) every ``log_every`` steps (scao/logging.py:89-121)."""

    def __init__(self, writer, log_every: int = 50, tag_prefix: str = "") -> None:
        self.writer = writer
        self.log_every = log_every
        self.tag_prefix = tag_prefix

    def __call__(self, metrics: MetricsDict) -> None:
        due, step = _due(metrics, self.log_every)
        if not due:
            return
        for k, v in metrics.items():
            if k == "step" or not isinstance(v, (bool, int, float)):
                continue
            x = float(v)
            if math.isnan(x):
                continue
            self.writer.add_scalar(self.tag_prefix + k, x, global_step=step)


class WandbLogger:
    """``wandb.log`` of the metrics every ``log_every`` steps; silently
    inactive without wandb (scao/logging.py:124-148)."""

    def __init__(self, log_every: int = 50) -> None:
        self.log_every = log_every

    def __call__(self, metrics: MetricsDict) -> None:
        due, step = _due(metrics, self.log_every)
        if not due:
            return
        try:
            import wandb  # type: ignore[import]
        except ImportError:
            return
        wandb.log({k: v for k, v in metrics.items() if k != "step"}, step=step)


def _l_norm(view):
    """Curvature-health figure of one Kronecker block: the int8 factor's
    scale * 127 (its absmax), else the Frobenius norm of the fp32 factor."""
    if view.use_int8_ema:
        return view.L_ema_scale * 127.0
    return float(view._fac(0).norm(p="fro").item())


def collect_metrics(optimizer) -> MetricsDict:
    """scao/logging.py:151-219: step, rank statistics, the mean curvature
    norm (per block-diagonal parameter the mean over its direct Kronecker
    blocks), precond_freq and the R1 warmup diagnostics."""
    step, ranks, norms = 0, [], []
    for st in optimizer.state.values():
        step = max(step, st.get("step", 0))
        prec = st.get("preconditioner")
        if prec is None:
            continue
        ranks.append(prec.k)
        if prec.use_block_diagonal:
            b = [_l_norm(c) for c in prec._blocks if c.use_kronecker]
            if b:
                norms.append(sum(b) / len(b))
        elif prec.use_kronecker:
            norms.append(_l_norm(prec._views[0]))
    m: MetricsDict = {"step": step}
    if ranks:
        m["scao/rank_mean"] = sum(ranks) / len(ranks)
        m["scao/rank_min"] = min(ranks)
        m["scao/rank_max"] = max(ranks)
        m["scao/layers"] = len(ranks)
    if norms:
        m["scao/L_norm_mean"] = sum(norms) / len(norms)
    m["scao/precond_freq"] = optimizer.param_groups[0].get("precond_freq", -1)
    ws = getattr(optimizer, "_warmup_scheduler", None)
    if ws is not None:
        m["scao/warmup_exited_early"] = ws.exited_early
        m["scao/actual_warmup_steps"] = ws.actual_warmup_steps
    return m
