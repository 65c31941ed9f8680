"""Arm: one prefill configuration (code/kva/kva.py:79-118 semantics).

Fills of a late layer's prefix rows [0, P) (P = N - tail):
  exact           no approximation (P = 0)
  proj            ridge projector x_i = W_i b + c_i (b = the row's split-layer input)
  identity        x_i = b for every late layer
  none            prefix rows never reach the layer (plain layer skip)
  oracle          the true layer inputs (all rows: reproduces exact prefill; a diagnostic)
  swiftkv         SwiftKV's distilled K/V for prefix rows; tail and decode exact
  swiftkv_native  SwiftKV as released: every row's late K/V from SwiftKV, queries through q_proj_swiftkv
  kvfold          attention layers' pre-RoPE K/V straight from the unit-RMS boundary state
  by_type         fill_by_type = {'attention': f, 'gdn': g}
Options: st (terminal-state corrections {layer: dS} added after a GDN layer's prefix fill), f1 (row 0 uses
its exact late inputs), context (projector input [b, c_{S-1}, .., c_{S-K}]), refresh (run layer R in full on
the filled prefix rows, then a refresh projector of split R+1), tail_bias_from / tail_bias_skip_last (the
tail's mean projector residual added to prefix fills), exact_part ('k' | 'v' from the true inputs),
rescale (knorm | kdir | vnorm oracle, ktail | vtail deployable) with rescale_skip_last, tail_from
('continuation': the tail is the scored rows).
"""
from __future__ import annotations

import dataclasses
from dataclasses import dataclass, field

ORACLE_RESCALE = ("knorm", "kdir", "vnorm")
TAIL_RESCALE = ("ktail", "vtail")
FILLS = ("exact", "proj", "identity", "none", "oracle", "swiftkv", "swiftkv_native", "kvfold", "by_type")
ENGINE_MIN_TAIL = 512   # a block-granular engine never runs a shorter exact tail


@dataclass
class Arm:
    """One prefill configuration. Every field past `name` is keyword-only in practice; the JSON arm specs use the
    same names."""
    name: str
    # where the approximation starts and how many exact rows end the prompt
    split: int | None = None
    tail: int = 0
    tail_from: str | None = None                 # "continuation": the tail is the scored continuation
    # how late layers see the prefix rows
    fill: str = "exact"
    fill_by_type: dict | None = None             # {"attention": fill, "gdn": fill}
    projector: object = None                     # ridge maps (fill "proj")
    kvfold: object = None                        # K/V fold maps (fill "kvfold")
    context: int = 0                             # mixer outputs of this many lower layers join the map input
    refresh: int | None = None                   # a late layer run in full on the filled rows ...
    refresh_projector: object = None             # ... feeding the maps fitted at refresh + 1
    # corrections
    st: dict | None = None                       # GDN terminal-state corrections {layer: dS}
    f1: bool = False                             # row 0 reads its exact late inputs
    tail_bias_from: int | None = None            # add the tail's mean map residual from this layer on
    tail_bias_skip_last: int = 0
    rescale: str | None = None                   # K or V norm rescale (see ORACLE_RESCALE / TAIL_RESCALE)
    rescale_skip_last: int = 0
    exact_part: str | None = None                # "k" | "v": that half from the true inputs (a diagnostic)
    meta: dict = field(default_factory=dict)     # the spec's remaining keys (select, sets, repair, ...)

    def __post_init__(self):
        if self.fill not in FILLS:
            raise ValueError(f"arm {self.name}: fill {self.fill!r} is not one of {FILLS}")
        if self.fill_by_type is not None:
            self.fill = "by_type"

    def prefix_len(self, n):
        """Rows [0, P) that are filled rather than run exactly."""
        return {"exact": 0, "swiftkv_native": n}.get(self.fill, max(0, n - self.tail))

    def fills(self):
        """Every fill this arm applies to some late layer."""
        return tuple(self.fill_by_type.values()) if self.fill_by_type else (self.fill,)

    def fill_of(self, layer_type):
        """The fill of a late layer of this type ('attn' or 'gdn'; by_type specs name attention 'attention')."""
        if self.fill_by_type is None:
            return self.fill
        key = "attention" if layer_type == "attn" else layer_type
        if key not in self.fill_by_type:
            raise ValueError(f"arm {self.name}: fill_by_type gives no fill for {key} layers")
        return self.fill_by_type[key]

    def uses(self, fill):
        return fill in self.fills()

    def uses_oracle(self):
        """The arm reads the true late-layer inputs (an oracle fill, exact_part or an oracle rescale)."""
        return self.exact_part is not None or self.rescale in ORACLE_RESCALE or "oracle" in self.fills()


def pop_split(n_layers):
    """POP's split: prefill prunes the last floor(L / 3) layers, S = L - floor(L / 3)."""
    return n_layers - n_layers // 3


def rounded_tail(n, base, block):
    """Tail length when the prefix boundary is rounded down to a block multiple (tail >= base)."""
    prefix = (n - base) // block * block if n > base else 0
    return n - prefix


def exclude_scored(arm, scored):
    """The arm with its tail statistics (ktail / vtail scale, tail bias) kept off the last `scored` rows."""
    changes = {}
    if scored > 0 and arm.rescale in TAIL_RESCALE:
        changes["rescale_skip_last"] = max(arm.rescale_skip_last, scored)
    if scored > 0 and arm.tail_bias_from is not None:
        changes["tail_bias_skip_last"] = max(arm.tail_bias_skip_last, scored)
    return dataclasses.replace(arm, **changes) if changes else arm
