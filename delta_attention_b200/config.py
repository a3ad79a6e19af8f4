"""Configuration knobs of the delta-attention plug-in.

Mirrors the hot-path fields of the reference's ``Config`` dataclass
(``delta_attention/config.py:9-78``) with the same names, defaults and
meaning, plus two fields the reference hard-codes:

* ``sink`` -- attention-sink tokens; the reference fixes 1024
  (``delta_attention/llama.py:415,543``).
* ``q_block`` -- query block of hip-attn's block-anchored window; the
  reference fixes 64 (``delta_attention/config.py:117,136``).

``delta_lambda`` keeps the reference's meaning: the integer anchor stride
(gamma), not a scale factor (``delta_attention/llama.py:651,673``).
The reference's config is built with ``argparse_dataclass``; this one is a
plain dataclass with an equivalent ``from_args`` helper.
"""

from __future__ import annotations

import argparse
import dataclasses
from dataclasses import dataclass, field
from typing import Iterable, List, Optional, Sequence


@dataclass
class Config:
    model_str: str = "meta-llama/Llama-3.1-8B-Instruct"
    attn_implementation: str = "window"      # [window, hip_attention, flash_attention_2]
    mode: str = "delta"                      # [delta, recompute, sparse-only]

    delta_lambda: int = 64                   # anchor stride gamma
    sliding_window: int = 2048               # window W
    sink: int = 1024                         # sink tokens S (reference hard-codes 1024)
    q_block: int = 64                        # block-anchored window granularity
    delta_grad_scale: float = 1.0            # training-only knob, carried for compatibility

    log_drift: bool = False                  # prefill drift telemetry (anchor-delta cosine)

    stride_policy: str = "fixed"             # [fixed, adaptive]
    gamma_min: int = 16
    gamma_max: int = 256
    adapt_chunk: int = 4096
    adapt_threshold: float = 0.95
    stride_trigger: str = "absolute"         # [absolute, relative]
    adapt_k: float = 2.0

    decode_mode: str = "dense"               # [dense, sparse, delta]
    gamma_dec: int = 32
    refresh_policy: str = "fixed"            # [fixed, drift, drift_rel]
    drift_threshold: float = 0.95
    drift_k: float = 2.0
    gamma_dec_max: int = 128

    max_new_tokens: int = 128

    @classmethod
    def from_args(cls, argv: Optional[Sequence[str]] = None) -> "Config":
        """Parse ``--field value`` flags for every field (bools are presence flags)."""
        ap = argparse.ArgumentParser()
        for f in dataclasses.fields(cls):
            if f.type in ("bool", bool):
                ap.add_argument(f"--{f.name}", action="store_true", default=f.default)
            else:
                typ = {"int": int, "float": float, "str": str}.get(str(f.type), str)
                ap.add_argument(f"--{f.name}", type=typ, default=f.default)
        return cls(**vars(ap.parse_args(argv)))


# Knobs the attention plug-in reads from ``model.config`` at call time
# (``delta_attention/config.py:87-93`` plus ``sink`` and ``q_block``).
PIPELINE_FIELDS = (
    "mode", "delta_lambda", "sliding_window", "sink", "q_block", "log_drift", "delta_grad_scale",
    "stride_policy", "gamma_min", "gamma_max", "adapt_chunk",
    "adapt_threshold", "stride_trigger", "adapt_k",
    "decode_mode", "gamma_dec", "refresh_policy", "drift_threshold",
    "drift_k", "gamma_dec_max",
)


def apply_pipeline_fields(config: Config, model_config) -> None:
    """Copy the pipeline knobs onto a model config object
    (``delta_attention/sample.py:303-304``, ``model_wrapper.py:22-42``)."""
    for name in PIPELINE_FIELDS:
        setattr(model_config, name, getattr(config, name))
    model_config.attn_implementation_original = config.attn_implementation
