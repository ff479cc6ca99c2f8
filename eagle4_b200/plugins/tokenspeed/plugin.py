"""TokenSpeed plugin entry point: registers the EAGLE_HARNESS drafter and the EAGLE-4 draft architecture when the
installed TokenSpeed carries the plugin contract (``eagle4_b200.plugins.tokenspeed.hooks``); otherwise registers
nothing and logs what is missing (reference ``eagle_harness/tokenspeed/plugin.py``)."""

from __future__ import annotations

import logging

log = logging.getLogger(__name__)

DRAFT_ARCHITECTURE = "LlamaForCausalLMEagle4"


def register() -> bool:
    from eagle4_b200.compat import check_for_registration

    if not check_for_registration("tokenspeed"):
        return False
    from tokenspeed.runtime.plugins.registry import register_drafter, register_model

    from eagle4_b200.plugins.tokenspeed.models import LlamaForCausalLMEagle4
    from eagle4_b200.plugins.tokenspeed.adapter import ALGORITHM, HarnessDrafter

    register_model(cls=LlamaForCausalLMEagle4, architectures=[DRAFT_ARCHITECTURE])
    register_drafter(algorithm=ALGORITHM, drafter_cls=HarnessDrafter, model_cls=LlamaForCausalLMEagle4,
                     captures_aux_hidden_states=True, uses_tree_layout=True)
    log.info("eagle4_b200: registered TokenSpeed drafter %s", ALGORITHM)
    return True
