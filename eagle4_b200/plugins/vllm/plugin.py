"""vLLM plugin entry point (entry-point group ``vllm.general_plugins``): registers the ``eagle_harness``
speculative method when the installed vLLM carries every hook of ``eagle4_b200.plugins.vllm.hooks.HOOK_MAP``;
otherwise registers nothing and logs what is missing (reference ``eagle_harness/vllm/plugin.py``)."""

from __future__ import annotations

import logging

log = logging.getLogger(__name__)


def register() -> bool:
    from eagle4_b200.compat import check_for_registration

    if not check_for_registration("vllm"):
        return False
    from vllm.v1.spec_decode.registry import register_speculative_method

    from eagle4_b200.plugins.vllm.adapter import METHOD, HarnessMethodSpec, HarnessSpeculator

    register_speculative_method(METHOD, HarnessMethodSpec, HarnessSpeculator)
    log.info("eagle4_b200: registered vLLM speculative method %s", METHOD)
    return True
