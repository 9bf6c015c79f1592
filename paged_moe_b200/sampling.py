"""Per-request sampling defaults (host side, pure Python).

Public functions with the reference's names and results
(pagedmoe/sampling.py: family_for :56, defaults_for :76, describe :110,
fill :121), pinned by tests/golden/sampling_defaults.json, which the
reference itself produced.

Resolution here is a stack of layers, lowest priority first:

    1. the model family's published serving recipe   (source "<family> family")
    2. the checkpoint's generation_config.json        (source "generation_config.json")

Each layer maps setting -> value; a higher layer replaces a lower one's value
but the setting keeps the position it first appeared at (the log line lists
settings in that order).  The merged result is then pruned of values that
switch a filter off, and of a repetition window without a penalty.  A
generation config that says do_sample false, or a resolved temperature of
zero or below, means greedy: no defaults at all.  At request time, whatever
the request body or a server flag sets wins over every layer.
"""

from __future__ import annotations

import json
import re
import sys
from dataclasses import dataclass
from pathlib import Path
from typing import Callable, Dict, List, Mapping, Optional, Tuple


@dataclass(frozen=True)
class Recipe:
    family: str
    pattern: "re.Pattern[str]"
    settings: Mapping[str, float]


def _r(family: str, regex: str, **settings) -> Recipe:
    return Recipe(family, re.compile(regex, re.I), settings)


# Published serving recipes, most specific pattern first (the first match
# wins).  The values are the ones callers of the reference resolve to, so they
# must not drift.  No recipe sets a presence penalty: over a 20-token window
# it punishes the indentation, quotes and keys that code legitimately repeats.
RECIPES: Tuple[Recipe, ...] = (
    _r("qwen", r"qwen[34]|qwen3_next|qwen3_5|qwen4_exp",
       temperature=0.6, top_p=0.95, top_k=20, repetition_penalty=1.05, repetition_context_size=64),
    _r("deepseek", r"deepseek", temperature=0.6, top_p=0.95, top_k=40),
    _r("glm", r"^glm|chatglm", temperature=0.6, top_p=0.95, top_k=40),
    _r("kimi", r"kimi|moonshot", temperature=0.6, top_p=0.95, top_k=40),
    _r("minimax", r"minimax", temperature=0.6, top_p=0.95, top_k=40),
    _r("gpt-oss", r"gpt[_-]?oss", temperature=1.0, top_p=1.0),
    _r("mistral", r"mistral|mixtral|magistral|devstral", temperature=0.15, top_p=0.9, top_k=40),
    _r("gemma", r"gemma", temperature=1.0, top_p=0.95, top_k=64),
    _r("llama", r"llama", temperature=0.6, top_p=0.9, top_k=40),
    _r("phi", r"phi[_-]?[34]|phi3|phi4", temperature=0.8, top_p=0.95, top_k=40),
    _r("granite", r"granite", temperature=0.6, top_p=0.9, top_k=40),
)

# The same table as (family, pattern, settings) triples.
FAMILIES = tuple((r.family, r.pattern, dict(r.settings)) for r in RECIPES)

# generation_config.json entries this layer reads, and the type each becomes
_CONFIG_TYPES: Dict[str, type] = {
    "temperature": float, "top_p": float, "top_k": int, "min_p": float, "repetition_penalty": float,
}

# server command-line flags that give a setting a default of their own
_SERVER_FLAGS: Dict[str, str] = {"temperature": "--temp", "top_p": "--top-p", "top_k": "--top-k",
                                 "min_p": "--min-p"}

# a value that leaves the sampler unchanged (the filter or penalty is off)
_SWITCHED_OFF: Dict[str, Callable[[float], bool]] = {
    "top_p": lambda v: v >= 1.0,
    "top_k": lambda v: v <= 0,
    "min_p": lambda v: v <= 0,
    "repetition_penalty": lambda v: v <= 0 or v == 1.0,
}

_GREEDY_SERVER = "none, the server's own defaults apply"


def family_for(model_type: str, name: str):
    """(family, settings) of the first recipe whose pattern occurs in the
    model type; failing that, in the checkpoint's folder name."""
    for text in (model_type, name):
        hit = next((r for r in RECIPES if text and r.pattern.search(text)), None)
        if hit is not None:
            return hit.family, dict(hit.settings)
    return None, {}


def _load_generation_config(model_dir: Optional[str]) -> dict:
    if not model_dir:
        return {}
    try:
        data = json.loads((Path(model_dir).expanduser() / "generation_config.json").read_text())
    except (OSError, ValueError):
        return {}
    return data if isinstance(data, dict) else {}


def _config_layer(gen: dict) -> Dict[str, float]:
    """The usable sampler entries of a generation config: present, not a
    bool, convertible to the sampler's type, and not negative."""
    layer: Dict[str, float] = {}
    for key, kind in _CONFIG_TYPES.items():
        raw = gen.get(key)
        if raw is None or isinstance(raw, bool):
            continue
        try:
            value = kind(raw)
        except (TypeError, ValueError):
            continue
        if value >= 0:
            layer[key] = value
    return layer


def defaults_for(model_dir: Optional[str], model_type: str = "") -> tuple:
    """(defaults, sources) for a checkpoint: each default setting, and for
    each the layer it came from."""
    gen = _load_generation_config(model_dir)
    if gen.get("do_sample") is False:
        return {}, {}
    family, recipe = family_for(model_type or "", Path(model_dir).name if model_dir else "")
    layers: List[Tuple[str, Mapping[str, float]]] = [
        (f"{family} family", recipe),
        ("generation_config.json", _config_layer(gen)),
    ]
    merged: Dict[str, Tuple[float, str]] = {}
    for source, layer in layers:
        for key, value in layer.items():
            merged[key] = (value, source)  # an existing key keeps its position
    if merged.get("temperature", (1.0, ""))[0] <= 0:
        return {}, {}
    kept = {k: vs for k, vs in merged.items() if not (k in _SWITCHED_OFF and _SWITCHED_OFF[k](vs[0]))}
    if "repetition_penalty" not in kept:
        kept.pop("repetition_context_size", None)
    return {k: v for k, (v, _) in kept.items()}, {k: s for k, (_, s) in kept.items()}


def describe(defaults: dict, sources: dict) -> str:
    """One log line: the settings grouped by their source, each group in the
    order its first setting appears ("temperature 0.6, top_k 20 (qwen family); ...")."""
    if not defaults:
        return _GREEDY_SERVER
    order: List[str] = []
    parts: Dict[str, List[str]] = {}
    for key, value in defaults.items():
        if key == "repetition_context_size":  # rides along with the penalty
            continue
        src = sources.get(key, "?")
        if src not in parts:
            order.append(src)
            parts[src] = []
        parts[src].append(f"{key} {value:g}")
    return "; ".join(", ".join(parts[src]) + f" ({src})" for src in order)


def _flag_given(flag: str, argv) -> bool:
    return any(arg == flag or arg.startswith(flag + "=") for arg in argv)


def fill(handler, body: dict, defaults: dict, argv=None) -> list:
    """Give `handler` (the server's request handler) every default that
    neither the request body nor a server flag sets; returns those keys."""
    argv = sys.argv if argv is None else argv

    def overridden(key: str) -> bool:
        if key in body:
            return True
        # a request that brings its own penalty keeps the server's window for it
        if key == "repetition_context_size" and "repetition_penalty" in body:
            return True
        flag = _SERVER_FLAGS.get(key)
        return flag is not None and _flag_given(flag, argv)

    applied = [key for key in defaults if not overridden(key)]
    for key in applied:
        setattr(handler, key, defaults[key])
    return applied
