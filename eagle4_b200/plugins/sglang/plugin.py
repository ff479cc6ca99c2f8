"""SGLang plugin entry point (entry-point group ``sglang.srt.plugins``).

``sglang.srt.plugins.load_plugins()`` calls :func:`register` once per process. It registers the EAGLE_HARNESS
speculative algorithm and the EAGLE-4 draft architecture and patches nothing. On an SGLang whose hooks differ from
``eagle4_b200.plugins.sglang.hooks.HOOKS`` it registers nothing and logs the mismatches (``eagle4_b200.compat``), so
``--speculative-algorithm EAGLE_HARNESS`` stays unknown and SGLang keeps working (reference
``eagle_harness/sglang/plugin.py:23-57``: same registration rule).
"""

from __future__ import annotations

import logging

log = logging.getLogger(__name__)

MODEL_PACKAGE = "eagle4_b200.plugins.sglang.models"
DRAFT_ARCHITECTURE = "LlamaForCausalLMEagle4"


def register() -> bool:
    """Register the algorithm and the draft model (idempotent); False when the installed SGLang lacks a hook."""
    from eagle4_b200.compat import check_for_registration

    if not check_for_registration("sglang"):
        return False
    from sglang.srt.models.registry import ModelRegistry
    from sglang.srt.speculative.spec_info import SpeculativeAlgorithm

    from eagle4_b200.plugins.sglang.adapter import ALGORITHM_NAME, HarnessSpecAlgo

    try:
        SpeculativeAlgorithm.from_string(ALGORITHM_NAME)
        return True  # already registered in this process
    except ValueError:
        pass
    if DRAFT_ARCHITECTURE not in ModelRegistry.get_supported_archs():
        ModelRegistry.register(MODEL_PACKAGE, strict=True)

    @SpeculativeAlgorithm.register(ALGORITHM_NAME, supports_overlap=True, spec_class=HarnessSpecAlgo)
    def _worker_class(server_args):
        from eagle4_b200.plugins.sglang.adapter import HarnessWorker

        return HarnessWorker

    log.info("eagle4_b200: registered speculative algorithm %s and models from %s", ALGORITHM_NAME, MODEL_PACKAGE)
    return True
