# SPDX-License-Identifier: Apache-2.0
"""Route table: which Sage3 config each (layer, denoising step) uses.

Same file format and matching rules as the reference
(src/vllm_qdq_plugin/sage3_attn/routing/route_table.py):

    {"default": "mxfp4",
     "rules": [{"layers": "20-39", "steps": "0-7", "config": "mixed_fp8qk_fp4pv"},
               {"steps": "0-7", "config": "sdpa"}]}

A rule's optional `layers` / `steps` are inclusive range strings ("0-7,9") or
single integers; `config` is a Sage3 config name or "sdpa" (full-precision
attention).  Rules are tried in order and the first whose present predicates
all hold wins; otherwise `default` (None when absent).  A predicate on a
dimension whose index is unknown (None) does not hold.  Every error in the
file is a ValueError at load time.
"""

from __future__ import annotations

import json

from ..sage3.api import ATTENTION_CONFIGS, REFERENCE_CONFIG_NAMES

SDPA_TOKEN = "sdpa"


def allowed_configs() -> set[str]:
    """Config names a route may name: every name the reference registers (so
    its route files load unchanged), this build's names, and "sdpa"."""
    return set(ATTENTION_CONFIGS) | set(REFERENCE_CONFIG_NAMES) | {SDPA_TOKEN}


def _parse_ranges(spec: str) -> set[int]:
    """"0-7,9,12-15" -> {0..7, 9, 12..15}; whitespace is ignored, "" is empty."""
    out: set[int] = set()
    for piece in spec.split(","):
        piece = piece.strip()
        if not piece:
            continue
        lo, sep, hi = piece.partition("-")
        try:
            a = int(lo.strip())
            b = int(hi.strip()) if sep else a
        except ValueError:
            raise ValueError(f"invalid range piece {piece!r} in {spec!r}") from None
        if b < a:
            raise ValueError(f"descending range {piece!r} in {spec!r}")
        out.update(range(a, b + 1))
    return out


def _range_field(rule: dict, field: str, idx: int) -> set[int] | None:
    if field not in rule:
        return None
    value = rule[field]
    if isinstance(value, bool) or not isinstance(value, (int, str)):
        raise ValueError(f"route rule {idx}: {field!r} must be a range string or an integer, "
                         f"got {type(value).__name__}")
    return _parse_ranges(str(value))


class _Rule:
    __slots__ = ("layers", "steps", "config")

    def __init__(self, layers: set[int] | None, steps: set[int] | None, config: str):
        self.layers, self.steps, self.config = layers, steps, config

    def matches(self, layer_idx: int | None, step_idx: int | None) -> bool:
        for wanted, got in ((self.layers, layer_idx), (self.steps, step_idx)):
            if wanted is not None and (got is None or got not in wanted):
                return False
        return True


class RouteTable:
    """Ordered, first-match-wins routing of attention configs."""

    def __init__(self, default: str | None, rules: list[_Rule]):
        self.default = default
        self.rules = rules

    @classmethod
    def from_json_file(cls, path: str) -> "RouteTable":
        with open(path) as f:
            data = json.load(f)
        if not isinstance(data, dict):
            raise ValueError(f"route file {path!r} must hold a JSON object, got {type(data).__name__}")
        allowed = allowed_configs()
        default = data.get("default")
        if default is not None and default not in allowed:
            raise ValueError(f"route file {path!r}: default {default!r} is not a known config")
        raw = data.get("rules", [])
        if not isinstance(raw, list):
            raise ValueError(f"route file {path!r}: 'rules' must be a list, got {type(raw).__name__}")
        rules = []
        for i, r in enumerate(raw):
            if not isinstance(r, dict):
                raise ValueError(f"route file {path!r}: rule {i} must be an object")
            if "config" not in r:
                raise ValueError(f"route file {path!r}: rule {i} has no 'config'")
            if r["config"] not in allowed:
                raise ValueError(f"route file {path!r}: rule {i} config {r['config']!r} is not a known config")
            rules.append(_Rule(_range_field(r, "layers", i), _range_field(r, "steps", i), r["config"]))
        return cls(default, rules)

    def resolve(self, layer_idx: int | None, step_idx: int | None) -> str | None:
        """The routed config name, or None to keep the impl's own config."""
        for rule in self.rules:
            if rule.matches(layer_idx, step_idx):
                return rule.config
        return self.default
