"""Which linear layers a `[quantize]` target selects (module names in, bool out).

The selection rule must pick exactly the modules the reference picks (byteprof/quant/select.py:18-59),
so the name patterns are the reference's: Bolmo's local encoder/decoder projections and MLPs plus the
encoder out_projection and decoder in_projection ("local"), and the transformer layers' attention and
MLP projections ("global"; OLMo 2's "blocks" use the same names). Embeddings, lm_head (except for
OLMo's "blocks+head"), the boundary predictor and the mLSTM gate projections are never selected.
"""

from __future__ import annotations

import re

BOLMO_TARGETS = ("none", "local", "global", "all")
OLMO_TARGETS = ("blocks", "blocks+head")
VALID_TARGETS = BOLMO_TARGETS + OLMO_TARGETS
VALID_SCHEMES = ("int8_wo", "int4_wo")

_LOCAL_LAYER = r"model\.local_(?:encoder|decoder)\.layers\.\d+\."
_LOCAL = re.compile(
    "^(?:" + _LOCAL_LAYER + r"(?:xlstm\.(?:q|k|v|ogate_preact|out_proj)|mlp\.(?:gate_proj|up_proj|down_proj))"
    r"|model\.local_encoder\.out_projection|model\.local_decoder\.in_projection)$")
_GLOBAL = re.compile(r"^model\.layers\.\d+\.(?:self_attn\.(?:q|k|v|o)_proj|mlp\.(?:gate_proj|up_proj|down_proj))$")


def group_of(module_name: str) -> str | None:
    """"local", "global" or None (never quantized)."""
    if _LOCAL.match(module_name):
        return "local"
    if _GLOBAL.match(module_name):
        return "global"
    return None


def should_quantize(module_name: str, target: str) -> bool:
    """Bolmo targets: none | local | global | all."""
    if target not in BOLMO_TARGETS:
        raise ValueError(f"Bolmo target must be one of {list(BOLMO_TARGETS)}, got {target!r}")
    g = group_of(module_name)
    return g is not None and target in ("all", g)


def olmo_group_of(module_name: str) -> str | None:
    """"blocks" for the transformer layers' linears, "head" for lm_head, else None."""
    if _GLOBAL.match(module_name):
        return "blocks"
    return "head" if module_name == "lm_head" else None


def olmo_should_quantize(module_name: str, target: str) -> bool:
    """OLMo 2 targets: none | blocks | blocks+head."""
    if target not in ("none",) + OLMO_TARGETS:
        raise ValueError(f"OLMo target must be one of {['none', *OLMO_TARGETS]}, got {target!r}")
    g = olmo_group_of(module_name)
    if g is None or target == "none":
        return False
    return g == "blocks" or target == "blocks+head"


def selects(target: str, group: str | None) -> bool:
    """Does `target` quantize a linear of this group (local, global, blocks, head)?"""
    if group is None or target == "none":
        return False
    allowed = {"local": ("local",), "global": ("global",), "all": ("local", "global"),
               "blocks": ("blocks",), "blocks+head": ("blocks", "head")}[target]
    return group in allowed
