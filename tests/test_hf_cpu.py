"""HuggingFace glue (host only): parameter split, scheduler, Trainer and
callback classes.  No step runs here (the optimizer needs CUDA tensors)."""
import pytest
import torch.nn as nn

transformers = pytest.importorskip("transformers")

from scao_b200 import SCAO  # noqa: E402
from scao_b200.integrations import huggingface as hf  # noqa: E402


class Tiny(nn.Module):
    def __init__(self):
        super().__init__()
        self.fc = nn.Linear(16, 32)
        self.LayerNorm = nn.LayerNorm(32)
        self.out = nn.Linear(32, 4, bias=False)


def _args(tmp_path):
    """The TrainingArguments fields the glue reads (TrainingArguments itself
    needs ``accelerate``, which this image lacks)."""
    from types import SimpleNamespace
    return SimpleNamespace(output_dir=str(tmp_path), learning_rate=3e-4, weight_decay=0.05,
                           warmup_steps=7, max_steps=50, lr_scheduler_type="cosine")


def test_get_scao_optimizer_groups(tmp_path):
    m = Tiny()
    opt, sched = hf.get_scao_optimizer(m, _args(tmp_path), scao_kwargs=dict(k_max=16))
    assert isinstance(opt, SCAO)
    g0, g1 = opt.param_groups
    names = {id(p): n for n, p in m.named_parameters()}
    assert {names[id(p)] for p in g0["params"]} == {"fc.weight", "out.weight"}
    assert {names[id(p)] for p in g1["params"]} == {"fc.bias", "LayerNorm.weight", "LayerNorm.bias"}
    assert g0["weight_decay"] == 0.05 and g1["weight_decay"] == 0.0
    assert g0["lr"] == pytest.approx(0.0)          # the scheduler's warmup starts at 0
    assert opt.defaults["warmup_steps"] == 7 and opt.defaults["k_max"] == 16
    sched.step()
    assert g0["lr"] > 0.0


def test_trainer_and_callback(tmp_path):
    assert hf.SCAOTrainer is not None and hf.SCAOMonitorCallback is not None
    m = Tiny()
    opt, _ = hf.get_scao_optimizer(m, _args(tmp_path))
    try:
        import accelerate  # noqa: F401
        args = transformers.TrainingArguments(output_dir=str(tmp_path), report_to=[])
        tr = hf.SCAOTrainer(model=m, args=args, scao_kwargs=dict(k_max=8))
        assert isinstance(tr.create_optimizer(), SCAO)
    except ImportError:
        pass
    cb = hf.SCAOMonitorCallback(opt)
    logs = {}
    cb.on_log(None, None, None, logs=logs)
    assert "global_norm_ema" in logs and "noise_std" in logs
