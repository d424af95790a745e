"""HuggingFace ``Trainer`` glue for scao_b200 (same entry points as
scao/integrations/huggingface.py:54-246 of the reference):

* ``get_scao_optimizer(model, training_args)`` -> (optimizer, lr scheduler),
  with the usual decay / no-decay parameter split;
* ``SCAOTrainer`` -- a ``Trainer`` whose optimizer is SCAO;
* ``SCAOMonitorCallback`` -- adds SCAO's rank / norm metrics to the logs.

``transformers`` is imported lazily; without it the two classes are None,
as in the reference.
"""
from __future__ import annotations

from typing import Any

NO_DECAY = ("bias", "LayerNorm.weight", "layer_norm.weight")


def _split_decay(model, no_decay_names):
    """Trainable parameters whose name contains a no-decay marker go to the
    zero-weight-decay group (scao/integrations/huggingface.py:96-108)."""
    decay, plain = [], []
    for name, p in model.named_parameters():
        if not p.requires_grad:
            continue
        (plain if any(nd in name for nd in no_decay_names) else decay).append(p)
    return decay, plain


def get_scao_optimizer(model, training_args, scao_kwargs: dict | None = None,
                       no_decay_names: tuple = NO_DECAY):
    """SCAO over ``model`` with ``training_args``' learning rate, weight decay
    and warmup, plus the Trainer's learning-rate scheduler
    (scao/integrations/huggingface.py:54-128)."""
    try:
        from transformers import get_scheduler
    except ImportError as e:
        raise ImportError("transformers is required for get_scao_optimizer") from e
    from ..optimizer import SCAO

    decay, plain = _split_decay(model, no_decay_names)
    groups = [{"params": decay, "weight_decay": training_args.weight_decay},
              {"params": plain, "weight_decay": 0.0}]
    kw: dict[str, Any] = dict(lr=training_args.learning_rate,
                              warmup_steps=int(getattr(training_args, "warmup_steps", 100)))
    kw.update(scao_kwargs or {})
    optimizer = SCAO(groups, **kw)
    total = getattr(training_args, "max_steps", -1)
    if total is None or total < 0:
        total = 10_000
    scheduler = get_scheduler(name=getattr(training_args, "lr_scheduler_type", "cosine"),
                              optimizer=optimizer,
                              num_warmup_steps=getattr(training_args, "warmup_steps", 0),
                              num_training_steps=total)
    return optimizer, scheduler


def _trainer_class():
    try:
        from transformers import Trainer
    except ImportError:
        return None

    class SCAOTrainer(Trainer):
        """``Trainer`` with SCAO as its optimizer; ``scao_kwargs`` are extra
        SCAO hyper-parameters (scao/integrations/huggingface.py:135-190)."""

        def __init__(self, *args, scao_kwargs: dict | None = None, **kwargs):
            self._scao_kwargs = dict(scao_kwargs or {})
            super().__init__(*args, **kwargs)

        def create_optimizer(self):
            if self.optimizer is None:
                self.optimizer, _ = get_scao_optimizer(self.model, self.args,
                                                       scao_kwargs=self._scao_kwargs)
            return self.optimizer

        def create_optimizer_and_scheduler(self, num_training_steps: int):
            self.create_optimizer()
            if self.lr_scheduler is None:
                try:
                    from transformers import get_scheduler
                    self.lr_scheduler = get_scheduler(
                        name=self.args.lr_scheduler_type, optimizer=self.optimizer,
                        num_warmup_steps=self.args.get_warmup_steps(num_training_steps),
                        num_training_steps=num_training_steps)
                except Exception:
                    super().create_optimizer_and_scheduler(num_training_steps)

    return SCAOTrainer


def _callback_class():
    try:
        from transformers import TrainerCallback
    except ImportError:
        return None

    class SCAOMonitorCallback(TrainerCallback):
        """Adds SCAO's numeric metrics (ranks, global grad-norm EMA, noise
        level, warmup flag) to every Trainer log
        (scao/integrations/huggingface.py:205-243)."""

        def __init__(self, optimizer, log_every: int | None = None) -> None:
            self.optimizer = optimizer
            self.log_every = log_every

        def on_log(self, args, state, control, logs=None, **kwargs):
            if logs is None:
                return
            metrics = self.optimizer.collect_metrics()
            logs.update({k: v for k, v in metrics.items()
                         if isinstance(v, (int, float)) and not isinstance(v, bool) and k != "step"})

    return SCAOMonitorCallback


SCAOTrainer = _trainer_class()
SCAOMonitorCallback = _callback_class()
