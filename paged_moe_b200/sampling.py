"""Per-request sampling defaults (host side, pure Python).

Same public functions and behaviour as the reference's pagedmoe/sampling.py
(family_for :56, defaults_for :76, describe :110, fill :121): a setting the
request leaves out comes from the checkpoint's generation_config.json, then
from the model family's serving recipe; anything the request or a server flag
sets wins, and a generation config with do_sample false keeps greedy decoding.
The family table holds the same published recipes as the reference
(sampling.py:34-47), so a request resolves to the same settings.
"""

from __future__ import annotations

import json
import re
import sys
from pathlib import Path
from typing import Optional

# (family, pattern, recipe); the first pattern that matches wins, specific
# patterns before general ones.  Recipes carry no presence penalty: applied
# over the last 20 tokens it hits the indentation, quotes and keys that code
# and tool calls legitimately repeat.
FAMILIES = (
    ("qwen", re.compile(r"qwen[34]|qwen3_next|qwen3_5|qwen4_exp", re.I),
     dict(temperature=0.6, top_p=0.95, top_k=20, repetition_penalty=1.05, repetition_context_size=64)),
    ("deepseek", re.compile(r"deepseek", re.I), dict(temperature=0.6, top_p=0.95, top_k=40)),
    ("glm", re.compile(r"^glm|chatglm", re.I), dict(temperature=0.6, top_p=0.95, top_k=40)),
    ("kimi", re.compile(r"kimi|moonshot", re.I), dict(temperature=0.6, top_p=0.95, top_k=40)),
    ("minimax", re.compile(r"minimax", re.I), dict(temperature=0.6, top_p=0.95, top_k=40)),
    ("gpt-oss", re.compile(r"gpt[_-]?oss", re.I), dict(temperature=1.0, top_p=1.0)),
    ("mistral", re.compile(r"mistral|mixtral|magistral|devstral", re.I), dict(temperature=0.15, top_p=0.9, top_k=40)),
    ("gemma", re.compile(r"gemma", re.I), dict(temperature=1.0, top_p=0.95, top_k=64)),
    ("llama", re.compile(r"llama", re.I), dict(temperature=0.6, top_p=0.9, top_k=40)),
    ("phi", re.compile(r"phi[_-]?[34]|phi3|phi4", re.I), dict(temperature=0.8, top_p=0.95, top_k=40)),
    ("granite", re.compile(r"granite", re.I), dict(temperature=0.6, top_p=0.9, top_k=40)),
)

# generation_config.json keys that are read, with the type the sampler takes
FILE_KEYS = (("temperature", float), ("top_p", float), ("top_k", int), ("min_p", float),
             ("repetition_penalty", float))

# server flags that carry a default of their own
CLI_FLAGS = {"temperature": "--temp", "top_p": "--top-p", "top_k": "--top-k", "min_p": "--min-p"}

# settings whose value means "filter off"; they are dropped from the defaults
_NO_OPS = {
    "top_p": lambda v: v >= 1.0,
    "top_k": lambda v: v <= 0,
    "min_p": lambda v: v <= 0,
    "repetition_penalty": lambda v: v == 1.0 or v <= 0,
}


def family_for(model_type: str, name: str):
    """(family, recipe) by model_type first, then by checkpoint folder name."""
    for text in (model_type, name):
        if not text:
            continue
        for fam, pattern, recipe in FAMILIES:
            if pattern.search(text):
                return fam, recipe
    return None, {}


def _read_generation_config(model_dir: Optional[str]) -> dict:
    if not model_dir:
        return {}
    path = Path(model_dir).expanduser() / "generation_config.json"
    try:
        data = json.loads(path.read_text())
    except (OSError, ValueError):
        return {}
    return data if isinstance(data, dict) else {}


def defaults_for(model_dir: Optional[str], model_type: str = "") -> tuple:
    """(defaults, sources) for a checkpoint; sources names where each came from."""
    gen = _read_generation_config(model_dir)
    if gen.get("do_sample") is False:
        return {}, {}
    fam, recipe = family_for(model_type or "", Path(model_dir).name if model_dir else "")
    out = dict(recipe)
    src = {key: f"{fam} family" for key in out}
    for key, cast in FILE_KEYS:
        raw = gen.get(key)
        if raw is None or isinstance(raw, bool):
            continue
        try:
            val = cast(raw)
        except (TypeError, ValueError):
            continue
        if val < 0:
            continue
        out[key] = val
        src[key] = "generation_config.json"
    if out.get("temperature", 1.0) <= 0:
        return {}, {}
    for key, is_noop in _NO_OPS.items():
        if key in out and is_noop(out[key]):
            del out[key]
            src.pop(key, None)
    if "repetition_penalty" not in out:
        out.pop("repetition_context_size", None)
        src.pop("repetition_context_size", None)
    return out, src


def describe(defaults: dict, sources: dict) -> str:
    """One log line: the settings grouped by where they came from."""
    if not defaults:
        return "none, the server's own defaults apply"
    groups: dict = {}
    for key, val in defaults.items():
        if key == "repetition_context_size":
            continue
        groups.setdefault(sources.get(key, "?"), []).append(f"{key} {val:g}")
    return "; ".join(f"{', '.join(items)} ({where})" for where, items in groups.items())


def fill(handler, body: dict, defaults: dict, argv=None) -> list:
    """Set on `handler` each default the request body leaves out; returns the keys set."""
    argv = sys.argv if argv is None else argv
    applied = []
    for key, val in defaults.items():
        if key in body:
            continue
        if key == "repetition_context_size" and "repetition_penalty" in body:
            continue
        flag = CLI_FLAGS.get(key)
        if flag and any(arg == flag or arg.startswith(flag + "=") for arg in argv):
            continue
        setattr(handler, key, val)
        applied.append(key)
    return applied
