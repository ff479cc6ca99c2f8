"""``--speculative-algorithm-config`` of ``EAGLE_HARNESS`` on TokenSpeed: the harness keys plus two of TokenSpeed's.

TokenSpeed hands the parsed JSON object to the drafter (``configure_algorithm``). Every harness key
(``core.config``) is read with the same strictness; TokenSpeed adds

* ``chain_width_table``: ``[[minimum batch size, verify width], ...]``, batch sizes increasing, widths >= 2: an
  explicit served chain schedule (chain intensity, serve mode); a table that starts at batch size 1 sets every width,
  so serve mode then needs no calibration data;
* ``sampled_proposals``: draw the tree's children instead of taking the top-k (serve mode).

The tree shape stays TokenSpeed's own flags (``--speculative-eagle-topk``, ``--speculative-num-steps``,
``--speculative-num-draft-tokens``). Serve mode (the default) needs ``data_path`` unless the chain table is complete:
TokenSpeed's round policy runs from calibrated tables only. The key names and the rules follow the reference
(``eagle_harness/tokenspeed/config.py:29-79``) so a TokenSpeed launch written for one reads the same here.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Any, Mapping, Optional, Tuple

from eagle4_b200.core.config import HarnessConfig, Mode, harness_config_from_dict
from eagle4_b200.core.limits import ComputeIntensity

ALGORITHM_NAME = "EAGLE_HARNESS"


@dataclass(frozen=True)
class TokenSpeedOptions:
    harness: HarnessConfig
    chain_width_table: Tuple[Tuple[int, int], ...] = ()
    sampled_proposals: bool = False

    @property
    def fully_scheduled(self) -> bool:
        """The chain table starts at batch size 1: it sets every width."""
        return bool(self.chain_width_table) and self.chain_width_table[0][0] == 1

    def chain_width(self, batch_size: int) -> Optional[int]:
        """The table's verify width for ``batch_size`` (None below its first entry or without a table)."""
        width = None
        for first, w in self.chain_width_table:
            if batch_size >= first:
                width = w
        return width


def _table(value: Any) -> Tuple[Tuple[int, int], ...]:
    if not isinstance(value, (list, tuple)):
        raise ValueError("chain_width_table is a list of [first batch size, verify width] pairs")
    out = []
    for entry in value:
        ok = (isinstance(entry, (list, tuple)) and len(entry) == 2
              and all(type(v) is int and v >= 1 for v in entry) and entry[1] >= 2
              and (not out or entry[0] > out[-1][0]))
        if not ok:
            raise ValueError(f"chain_width_table entry {entry!r}: batch sizes must be positive and increasing, widths "
                             "at least 2")
        out.append((int(entry[0]), int(entry[1])))
    return tuple(out)


def parse_algorithm_config(algorithm_config: Optional[Mapping[str, Any]]) -> TokenSpeedOptions:
    """The options of a launch (None reads as ``{}``); unknown keys and modes TokenSpeed cannot serve raise."""
    values = dict(algorithm_config or {})
    sampled = values.pop("sampled_proposals", False)
    if type(sampled) is not bool:
        raise ValueError(f"sampled_proposals must be true or false (found {sampled!r})")
    table = _table(values.pop("chain_width_table", ()))
    opts = TokenSpeedOptions(harness_config_from_dict(values), table, sampled)
    h = opts.harness
    if sampled and h.mode is not Mode.SERVE:
        raise ValueError("sampled_proposals is a serve-mode option")
    if h.mode is Mode.CALIBRATE and not h.data_path:
        raise ValueError("calibrate mode writes under data_path: set it")
    if table and (h.intensity is not ComputeIntensity.CHAIN or h.mode is not Mode.SERVE):
        raise ValueError("chain_width_table schedules served chains: it needs serve mode and chain_intensity")
    if h.mode is Mode.SERVE and not opts.fully_scheduled and not h.data_path:
        raise ValueError("serve mode on TokenSpeed prices rounds from calibration tables only: set data_path, give "
                         "chain_intensity a chain_width_table starting at batch size 1, or use {\"mode\": \"static\"} "
                         "for a fixed tree")
    return opts
