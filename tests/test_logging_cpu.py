"""Metrics sinks and collection (scao/logging.py) on the host: output format,
logging cadence, and the metric keys over preconditioner views of a host plan."""
import types

import torch

from scao_b200 import logging as slog
from scao_b200.plan import Plan
from scao_b200.preconditioner import PrecondView


def test_console_logger_format_and_cadence(capsys):
    log = slog.ConsoleLogger(log_every=10, prefix="[X]")
    log({"step": 3, "a": 1.0})
    assert capsys.readouterr().out == ""
    log({"step": 20, "a": 0.123456, "b": 7, "c": True})
    assert capsys.readouterr().out == "[X] step=20  a=0.1235  b=7  c=True\n"


def test_tensorboard_logger_scalars():
    seen = []
    w = types.SimpleNamespace(add_scalar=lambda tag, x, global_step: seen.append((tag, x, global_step)))
    slog.TensorBoardLogger(w, log_every=5, tag_prefix="t/")(
        {"step": 10, "r": 2, "f": float("nan"), "ok": True, "s": "text"})
    assert seen == [("t/r", 2.0, 10), ("t/ok", 1.0, 10)]


def test_wandb_logger(monkeypatch):
    import sys
    seen = []
    monkeypatch.setitem(sys.modules, "wandb",
                        types.SimpleNamespace(log=lambda d, step: seen.append((d, step))))
    slog.WandbLogger(log_every=2)({"step": 3, "a": 1.0})
    slog.WandbLogger(log_every=2)({"step": 4, "a": 1.0})
    assert seen == [({"a": 1.0}, 4)]


def test_collect_metrics_keys_and_values():
    g = dict(max_precond_dim=48, k_min=4, k_max=8, epsilon_sparse=0.05, rho=0.999,
             precond_freq=10)
    ps = [torch.zeros(32, 24), torch.zeros(96, 32), torch.zeros(16)]
    plan = Plan(ps, [g] * 3, torch.device("cpu"), True)
    state = {i: {"step": 5 + i, "preconditioner": PrecondView(plan, i, g)} for i in range(3)}
    ws = types.SimpleNamespace(exited_early=False, actual_warmup_steps=100)
    opt = types.SimpleNamespace(state=state, param_groups=[g], _warmup_scheduler=ws)
    m = slog.collect_metrics(opt)
    assert list(m) == ["step", "scao/rank_mean", "scao/rank_min", "scao/rank_max", "scao/layers",
                       "scao/L_norm_mean", "scao/precond_freq", "scao/warmup_exited_early",
                       "scao/actual_warmup_steps"]
    assert m["step"] == 7 and m["scao/layers"] == 3 and m["scao/rank_min"] == 1
    # int8 factors start at 1e-4 * I: absmax 1e-4 for every block
    assert abs(m["scao/L_norm_mean"] - 1e-4) < 1e-9
    assert m["scao/precond_freq"] == 10
