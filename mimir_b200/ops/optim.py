"""Fused multi-tensor AdamATan2 (+ decoupled weight decay, + EMA) step.

Reference math (``src/mimir/model/adam_atan2.py:105-132``), per parameter ``p`` with
gradient ``g``, step ``t`` and learning rate ``lr`` (times its per-parameter scale):

    p   *= 1 - lr * wd
    m    = lerp(m, g, 1 - b1)
    v    = b2 * v + (1 - b2) * g^2
    p   -= lr / (1 - b1^t) * atan2(m, sqrt(v) / sqrt(1 - b2^t))
    ema  = lerp(ema, p, 1 - ema_decay)

The CUDA kernel walks a device table of tensor chunks so one launch updates every
parameter of a group (fp32 or bf16 params/moments; fp32 EMA).
"""
from __future__ import annotations

from mimir_b200.ops._ext import ext


def adam_atan2_multi(params, grads, exp_avgs, exp_avg_sqs, emas, lrs, bias_corr1, bias_corr2_sqrt, beta1, beta2,
                     weight_decay, ema_decay):
    """One fused step over parallel tensor lists (``exp_avgs``/``emas`` may be ``None``).

    ``lrs`` are per-tensor learning rates (lr times its module scale); ``bias_corr1`` is
    ``1 - beta1^t`` and ``bias_corr2_sqrt`` is ``sqrt(1 - beta2^t)`` at the new step ``t``.
    """
    ext().adam_atan2_multi(params, grads, exp_avgs, exp_avg_sqs, emas, [float(x) for x in lrs],
                           [float(x) for x in bias_corr1], [float(x) for x in bias_corr2_sqrt], float(beta1),
                           float(beta2), float(weight_decay), float(ema_decay if ema_decay is not None else 0.0))
