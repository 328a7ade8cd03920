# SPDX-License-Identifier: Apache-2.0
"""Route table: which Sage3 config each (layer, denoising step) uses.

The file format is the reference's interface
(src/vllm_qdq_plugin/sage3_attn/routing/route_table.py:1-20), so its route
files load unchanged:

    {"default": "mxfp4",
     "rules": [{"layers": "20-39", "steps": "0-7", "config": "mixed_fp8qk_fp4pv"},
               {"steps": "0-7", "config": "sdpa"}]}

`layers` / `steps` are optional and written as inclusive ranges ("0-7,9") or
a bare integer; `config` names a Sage3 config or "sdpa" (full-precision
attention).  The first rule whose present fields all contain the call's
(layer, step) decides; otherwise `default` (None when absent).  An unknown
index (None) is contained in no range.

Here each range field becomes a sorted list of disjoint closed intervals
(membership by binary search), each rule one compiled predicate over
(layer, step), and the whole document is checked by one schema walk that
reports the path of the first offending field, e.g. ``rules[2].layers``.
"""

from __future__ import annotations

import bisect
import json
from typing import Callable

from ..sage3.api import ATTENTION_CONFIGS, REFERENCE_CONFIG_NAMES

SDPA_TOKEN = "sdpa"

Predicate = Callable[[int | None, int | None], bool]


def route_vocabulary() -> frozenset[str]:
    """Names a route may target: every config the reference registers (so its
    route files load unchanged), this build's names, and "sdpa"."""
    return frozenset(ATTENTION_CONFIGS) | frozenset(REFERENCE_CONFIG_NAMES) | {SDPA_TOKEN}


class IntervalSet:
    """A set of integers held as sorted, disjoint, non-adjacent [lo, hi] pairs."""

    __slots__ = ("_lo", "_hi")

    def __init__(self, pairs: list[tuple[int, int]]):
        merged: list[list[int]] = []
        for lo, hi in sorted(pairs):
            if merged and lo <= merged[-1][1] + 1:
                merged[-1][1] = max(merged[-1][1], hi)
            else:
                merged.append([lo, hi])
        self._lo = [p[0] for p in merged]
        self._hi = [p[1] for p in merged]

    @classmethod
    def parse(cls, spec: str | int) -> "IntervalSet":
        """"0-7,9,12-15" or 9 -> the set; blanks are ignored, "" is empty.
        Raises ValueError on anything that is not an integer or an ascending
        "a-b" pair."""
        if isinstance(spec, int):
            return cls([(spec, spec)])
        pairs = []
        for token in (t.replace(" ", "") for t in spec.split(",")):
            if not token:
                continue
            # a leading '-' would be a negative number, which no index takes
            cut = token.find("-", 1)
            ends = (token, token) if cut < 0 else (token[:cut], token[cut + 1:])
            if not all(e.isdigit() for e in ends):
                raise ValueError(f"{token!r} is neither an integer nor an 'a-b' range")
            lo, hi = int(ends[0]), int(ends[1])
            if hi < lo:
                raise ValueError(f"range {token!r} runs backwards")
            pairs.append((lo, hi))
        return cls(pairs)

    def intervals(self) -> list[tuple[int, int]]:
        return list(zip(self._lo, self._hi))

    def __contains__(self, x: object) -> bool:
        if not isinstance(x, int):
            return False
        i = bisect.bisect_right(self._lo, x) - 1
        return i >= 0 and x <= self._hi[i]

    def __iter__(self):
        for lo, hi in zip(self._lo, self._hi):
            yield from range(lo, hi + 1)

    def __eq__(self, other: object) -> bool:
        if isinstance(other, IntervalSet):
            return self.intervals() == other.intervals()
        if isinstance(other, (set, frozenset)):
            return set(self) == other
        return NotImplemented


def _compile(layers: IntervalSet | None, steps: IntervalSet | None) -> Predicate:
    """One predicate over (layer, step); an absent field accepts everything."""
    if layers is None and steps is None:
        return lambda layer, step: True
    if steps is None:
        return lambda layer, step: layer in layers
    if layers is None:
        return lambda layer, step: step in steps
    return lambda layer, step: layer in layers and step in steps


def _check_document(doc: object, vocab: frozenset[str]) -> tuple[str | None, list[tuple[Predicate, str]]]:
    """Validate a parsed route file and compile it.  Raises ValueError naming
    the path of the first field that breaks the schema."""

    def fail(where: str, why: str):
        raise ValueError(f"{where}: {why}")

    def config_name(value: object, where: str) -> str:
        if not isinstance(value, str) or value not in vocab:
            fail(where, f"{value!r} is not a Sage3 config name or {SDPA_TOKEN!r}")
        return value

    def range_field(value: object, where: str) -> IntervalSet:
        if isinstance(value, bool) or not isinstance(value, (int, str)):
            fail(where, f"expected a range string or an integer, got {type(value).__name__}")
        try:
            return IntervalSet.parse(value)
        except ValueError as e:
            fail(where, str(e))

    if not isinstance(doc, dict):
        fail("<root>", f"expected a JSON object, got {type(doc).__name__}")
    default = None if doc.get("default") is None else config_name(doc["default"], "default")
    rules = doc.get("rules", [])
    if not isinstance(rules, list):
        fail("rules", f"expected a list, got {type(rules).__name__}")
    compiled = []
    for i, rule in enumerate(rules):
        where = f"rules[{i}]"
        if not isinstance(rule, dict):
            fail(where, f"expected an object, got {type(rule).__name__}")
        if "config" not in rule:
            fail(where, "missing 'config'")
        target = config_name(rule["config"], f"{where}.config")
        fields = {f: range_field(rule[f], f"{where}.{f}") if f in rule else None for f in ("layers", "steps")}
        compiled.append((_compile(fields["layers"], fields["steps"]), target))
    return default, compiled


class RouteTable:
    """Ordered, first-match-wins routing of attention configs."""

    def __init__(self, default: str | None, routes: list[tuple[Predicate, str]]):
        self.default = default
        self._routes = tuple(routes)

    @classmethod
    def from_json_file(cls, path: str) -> "RouteTable":
        with open(path) as f:
            doc = json.load(f)
        try:
            default, routes = _check_document(doc, route_vocabulary())
        except ValueError as e:
            raise ValueError(f"route file {path!r}: {e}") from None
        return cls(default, routes)

    def __len__(self) -> int:
        """Number of rules (the default is not counted)."""
        return len(self._routes)

    def resolve(self, layer_idx: int | None, step_idx: int | None) -> str | None:
        """The routed config name, or None to keep the impl's own config."""
        return next((cfg for matches, cfg in self._routes if matches(layer_idx, step_idx)), self.default)
