"""The training YAML of the reference (chessdecoder/train/config.yaml) as the
fused step's configuration.

* ``model:`` (config.yaml:11-20) -> ModelConfig;
* ``training:`` (:22-33) -> learning_rate, weight_decay,
  gradient_accumulation_steps (``TrainStep.grad_accum``, used by
  ``step_accumulated`` / the caller's loop); ``use_amp`` is accepted and has
  no effect (the step always runs bf16 operands with fp32 accumulation and
  fp32 master weights, which needs no loss scaling); device, checkpoint and
  logging keys belong to the caller's loop;
* ``loss:`` (:35-39) -> the move / board / WL / D loss weights;
* an optional ``kernels:`` section of this package: ``fp8`` (the fp8 recipe
  for the backbone linears), ``moe_experts`` / ``moe_capacity`` (the MoE
  variant), ``max_norm`` (the clip norm, 10.0 as train.py:249).

Keys this file does not know are ignored, as the reference's loop ignores
keys it does not read.
"""
from __future__ import annotations

from typing import Union

from .engine import ModelConfig, TrainStep
from . import vocab as V

_MODEL_KEYS = ("embed_dim", "num_heads", "num_layers", "max_seq_len", "d_ff", "n_buckets", "wl_sigma",
               "value_hidden_size", "num_fourier_freq")


def load_train_config(src: Union[str, dict]) -> dict:
    """The parsed YAML (a path) or the dict itself."""
    if isinstance(src, dict):
        return src
    import yaml
    with open(src) as f:
        return yaml.safe_load(f)


def model_config(conf: dict) -> ModelConfig:
    m = conf.get("model", {})
    k = conf.get("kernels", {}) or {}
    kw = {key: m[key] for key in _MODEL_KEYS if key in m}
    return ModelConfig(vocab_size=V.vocab_size, moe_experts=int(k.get("moe_experts", 0)),
                       moe_capacity=float(k.get("moe_capacity", 1.25)), **kw)


def step_from_config(src: Union[str, dict], device="cuda", seed: int = 0, state_dict=None) -> TrainStep:
    """A TrainStep configured as the YAML says (see the module docstring)."""
    conf = load_train_config(src)
    t = conf.get("training", {}) or {}
    lw = conf.get("loss", {}) or {}
    k = conf.get("kernels", {}) or {}
    weights = (float(lw.get("move_weight", 5.0)), float(lw.get("board_weight", 1.0)),
               float(lw.get("wl_weight", 1.0)), float(lw.get("d_weight", 1.0)))
    step = TrainStep(model_config(conf), device=device, seed=seed, lr=float(t.get("learning_rate", 1e-4)),
                     weight_decay=float(t.get("weight_decay", 0.1)), max_norm=float(k.get("max_norm", 10.0)),
                     loss_weights=weights, state_dict=state_dict, fp8=bool(k.get("fp8", False)))
    step.grad_accum = int(t.get("gradient_accumulation_steps", 1))
    return step
