"""The SGLang API the SGLang adapter is written against (hook-carrying SGLang builds, ``sglang>=0.5.23.dev0``).

The host attribute names and parameter lists are SGLang's interface and so are the same as the reference's table
(``eagle_harness/sglang/hooks.py:84-180``); the owners are this package's adapter classes.
"""

from __future__ import annotations

from typing import List

from eagle4_b200.plugins.contract import CALL, FIELD, OVERRIDE, Hook, override_mismatches, problems

_ALGO = "sglang.srt.speculative.spec_registry:CustomSpecAlgo"
_WORKER = "sglang.srt.speculative.eagle_worker_v2:EAGLEWorkerV2"
_DRAFT = "sglang.srt.speculative.eagle_worker_v2:EagleDraftWorker"
_SPEC_INPUT = "sglang.srt.speculative.spec_info:SpecInput"
_VERIFY_INPUT = "sglang.srt.speculative.eagle_info:EagleVerifyInput"
_EXT = "sglang.srt.layers.attention.linear.verify_extension:LinearAttnVerifyExtension"
_GRAPH_INFO = "sglang.srt.model_executor.runner.decode_graph_variants:DecodeGraphRunnerInfo"
_COMMON = "sglang.srt.speculative.eagle_worker_common"
_LOGITS = "sglang.srt.layers.logits_processor:LogitsProcessor"

MY_ALGO = "eagle4_b200.plugins.sglang.adapter:HarnessSpecAlgo"
MY_WORKER = "eagle4_b200.plugins.sglang.adapter:HarnessWorker"
MY_DRAFT = "eagle4_b200.plugins.sglang.adapter:HarnessDraftWorker"
MY_GDN = "eagle4_b200.plugins.sglang.adapter:GdnTreeVerify"
MY_MAMBA = "eagle4_b200.plugins.sglang.adapter:Mamba2TreeVerify"
MY_VERIFY_INPUT = "eagle4_b200.plugins.sglang.adapter:HarnessVerifyInput"

CONV_ARGS = ("layer", "mixed_qkv", "conv_states", "cache_indices", "intermediate_conv_window",
             "intermediate_state_indices")
RECURRENT_ARGS = ("layer", "query", "key", "value", "a", "b", "ssm_states", "cache_indices", "query_start_loc",
                  "intermediate_states", "intermediate_state_indices")
RUN_VERIFY_ARGS = ("batch", "target_worker", "req_to_token_pool", "token_to_kv_pool_allocator", "plan_stream",
                   "plan_stream_ctx", "topk", "num_draft_tokens", "device", "metadata_ready_pre_pad",
                   "finalize_tree_path", "grammar_barrier", "accept_step")
ACCEPT_INPUT = ("verify_input", "next_token_ids", "next_token_logits", "hidden_states", "seq_lens",
                "req_pool_indices", "out_cache_loc", "can_run_cuda_graph")
ACCEPT_RESULT = ("next_token_ids", "accept_lens", "accept_index", "new_seq_lens", "bonus_tokens", "hidden_states")
WORKER_INIT = ("server_args", "gpu_id", "nccl_port", "target_worker")

HOOKS = (
    Hook("sglang.srt.speculative.spec_info:SpeculativeAlgorithm.register", ("name", "supports_overlap", "spec_class")),
    Hook("sglang.srt.speculative.spec_info:SpeculativeAlgorithm.from_string", ("name",)),
    Hook(f"{_ALGO}.is_eagle", (), OVERRIDE, MY_ALGO),
    Hook(f"{_ALGO}.uses_aux_hidden_states", (), OVERRIDE, MY_ALGO),
    Hook(f"{_ALGO}.is_eagle3", (), OVERRIDE, MY_ALGO),
    Hook(f"{_ALGO}.handle_server_args", ("server_args",), OVERRIDE, MY_ALGO),
    Hook(f"{_ALGO}.supports_mm_inputs", (), OVERRIDE, MY_ALGO),
    Hook(f"{_ALGO}.req_to_token_extra_len", ("page_size",), OVERRIDE, MY_ALGO),
    Hook("sglang.srt.arg_groups.fields.spec:Spec.speculative_algorithm_config", (), FIELD),
    Hook(f"{_ALGO}.create_decode_graph_variants", ("info",), OVERRIDE, MY_ALGO),
    Hook(f"{_ALGO}.max_verify_batch_size", (), OVERRIDE, MY_ALGO, optional=True),
    Hook(f"{_GRAPH_INFO}.is_draft_worker", (), FIELD),
    Hook(f"{_GRAPH_INFO}.device", (), FIELD),
    Hook(f"{_ALGO}.create_linear_attn_verify_extension", ("state",), OVERRIDE, MY_ALGO),
    Hook(f"{_EXT}.init_cuda_graph_state", ("max_bs", "max_num_tokens"), OVERRIDE, MY_GDN),
    Hook(f"{_EXT}.begin_forward", ("layout", "in_graph"), OVERRIDE, MY_GDN),
    Hook(f"{_EXT}.reads_strided_inputs", (), OVERRIDE, MY_GDN),
    Hook(f"{_EXT}.conv_update", CONV_ARGS, OVERRIDE, MY_GDN),
    Hook(f"{_EXT}.recurrent_update", RECURRENT_ARGS, OVERRIDE, MY_GDN),
    Hook(f"{_EXT}.commit_state", ("state", "state_indices", "record_indices", "commit_steps", "parent"), OVERRIDE,
         MY_GDN, optional=True),
    Hook(f"{_EXT}.init_cuda_graph_state", ("max_bs", "max_num_tokens"), OVERRIDE, MY_MAMBA),
    Hook(f"{_EXT}.begin_forward", ("layout", "in_graph"), OVERRIDE, MY_MAMBA),
    Hook(f"{_EXT}.conv_update", CONV_ARGS, OVERRIDE, MY_MAMBA),
    Hook(f"{_SPEC_INPUT}.greedy_tokens_only", (), FIELD),
    Hook("sglang.srt.layers.logits_processor:LogitsProcessorOutput.next_token_ids", (), FIELD),
    # the candidate-logits processor of the draft's prefill path (plugins.candidate_logits)
    Hook(f"{_LOGITS}._get_logits", ("hidden_states", "lm_head", "logits_metadata", "embedding_bias",
                                    "use_logits_buffer"), OVERRIDE, optional=True),
    Hook(f"{_LOGITS}._copy_logits_to_buffer", ("logits", "logits_metadata", "use_buffer"), optional=True),
    Hook(f"{_VERIFY_INPUT}.prepared_out_cache_loc", (), FIELD),
    Hook(f"{_SPEC_INPUT}.flashinfer_verify_variant", ("bs", "num_tokens", "q_dtype", "kv_dtype", "head_dim"),
         OVERRIDE, MY_VERIFY_INPUT),
    Hook(f"{_COMMON}:run_eagle_verify", RUN_VERIFY_ARGS),
    Hook(f"{_COMMON}:run_eagle_verify", ("sampling_step",), CALL, optional=True),
    Hook(f"{_COMMON}:VerifyAcceptInput", ACCEPT_INPUT),
    Hook(f"{_COMMON}:VerifyAcceptResult", ACCEPT_RESULT),
    Hook(f"{_WORKER}.__init__", WORKER_INIT),
    Hook(f"{_WORKER}.create_draft_worker", WORKER_INIT, OVERRIDE, MY_WORKER),
    Hook(f"{_WORKER}.init_attention_backends", (), OVERRIDE, MY_WORKER),
    Hook(f"{_WORKER}._build_trivial_verify_input", ("batch",), OVERRIDE, MY_WORKER),
    Hook(f"{_WORKER}.forward_batch_generation", ("batch", "on_publish", "grammar_barrier", "pp_proxy_tensors"),
         OVERRIDE, MY_WORKER),
    Hook(f"{_DRAFT}.__init__", WORKER_INIT),
    Hook(f"{_DRAFT}.init_attention_backend", (), OVERRIDE, MY_DRAFT),
    Hook(f"{_DRAFT}._capture_cuda_graphs", (), OVERRIDE, MY_DRAFT),
)


def hook_problems() -> List[str]:
    return problems(HOOKS)


def adapter_problems() -> List[str]:
    """This package's overrides whose signatures differ from the table (checked without SGLang)."""
    return override_mismatches(HOOKS)
