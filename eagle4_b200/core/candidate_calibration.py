"""Offline-measured crossover of the candidate top-k paths (reference ``eagle_harness/core/candidate_calibration.py``).

``<data_path>/candidate_topk.json`` = ``{"identity": {...}, "max_single_pass_elements": n}``: the score count (rows x
candidates) up to which the one-pass top-k kernel beats the two-stage radix select on this exact setup. The identity
(device, torch version, dtype, vocabulary shard, candidate count) must match exactly, else the default dispatch
stays; nothing is timed at startup. A matching file with a malformed limit is an error. The reference's key name
``max_triton_elements`` is read as well, so its files load.
"""

import json
from pathlib import Path
from typing import Any, Mapping, Optional

FILE = "candidate_topk.json"


def load_candidate_crossover(data_path, identity: Mapping[str, Any]) -> Optional[int]:
    if data_path is None:
        return None
    path = Path(data_path) / FILE
    if not path.is_file():
        return None
    profile = json.loads(path.read_text())
    if profile.get("identity") != dict(identity):
        return None
    limit = profile.get("max_single_pass_elements", profile.get("max_triton_elements"))
    if type(limit) is not int or limit < 0:
        raise ValueError(f"{path}: the candidate top-k crossover {limit!r} is not a positive element count")
    return limit


def save_candidate_crossover(data_path, identity: Mapping[str, Any], limit: int) -> str:
    if type(limit) is not int or limit < 0:
        raise ValueError(f"the crossover must be a non-negative int, got {limit!r}")
    path = Path(data_path) / FILE
    path.parent.mkdir(parents=True, exist_ok=True)
    path.write_text(json.dumps({"identity": dict(identity), "max_single_pass_elements": limit}, indent=1))
    return str(path)
