"""End-to-end checking tools: greedy parity with fp32 arbitration (``parity``) and per-request stop conditions under
batched speculation (``stop_check``). Both talk to a running ``eagle4_b200.serve`` or drive the engine in-process."""
