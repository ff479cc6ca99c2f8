"""The EAGLE_HARNESS algorithm inside SGLang (hook-carrying SGLang builds): algorithm hooks, the GDN / Mamba2 tree
verify extensions, the verify attention variant and the cost-model worker.

SGLang keeps its scheduler, pools, prefill and target model; this adapter supplies what the reference's SGLang
package does (``eagle_harness/sglang/algorithm.py``, ``worker.py``, ``gdn_tree_verify.py``, ``mamba2_tree_verify.py``,
``verify_input.py``), built on this package's pieces: the round policy (cost model + live costs), the draft tree, the
sm_100a tree kernels (conv1d / gated delta rule / Mamba2 over the verify forest, tree attention, fused accept).

Every SGLang class is looked up at import and subclassed when present; without SGLang the classes subclass
``object`` so the module imports and the override signatures can be checked against the hook table
(``eagle4_b200.plugins.sglang.hooks``).
"""

from __future__ import annotations

import logging
from functools import cached_property
from typing import List, Optional

import torch

from eagle4_b200 import ops
from eagle4_b200.core.config import HarnessConfig, parse_harness_config
from eagle4_b200.core.limits import check_shape, req_to_token_span, verify_buckets
from eagle4_b200.plugins.common import GdnShape, TreeVerifyRows, accept_greedy_rows, gdn_conv, gdn_recurrence, host_base

log = logging.getLogger(__name__)

ALGORITHM_NAME = "EAGLE_HARNESS"
DEFAULT_TREE_SHAPE = (12, 4, 16)  # --speculative-num-steps, --speculative-eagle-topk, --speculative-num-draft-tokens

_CustomSpecAlgo = host_base("sglang.srt.speculative.spec_registry:CustomSpecAlgo")
_Extension = host_base("sglang.srt.layers.attention.linear.verify_extension:LinearAttnVerifyExtension")
_SpecInput = host_base("sglang.srt.speculative.eagle_info:EagleVerifyInput")
_Worker = host_base("sglang.srt.speculative.eagle_worker_v2:EAGLEWorkerV2")
_DraftWorker = host_base("sglang.srt.speculative.eagle_worker_v2:EagleDraftWorker")


def _spec_config_text() -> Optional[str]:
    try:
        from sglang.srt.runtime_context import get_spec

        return get_spec().speculative_algorithm_config
    except ImportError:
        return None


class HarnessSpecAlgo(_CustomSpecAlgo):
    """Algorithm-level hooks (one instance per process)."""

    @cached_property
    def config(self) -> HarnessConfig:
        return parse_harness_config(_spec_config_text())

    # EAGLE-family membership: own draft KV pool, target embedding shared, aux hidden states captured
    def is_eagle(self) -> bool:
        return True

    def uses_aux_hidden_states(self) -> bool:
        return True

    def is_eagle3(self) -> bool:
        return False

    def supports_mm_inputs(self) -> bool:
        return False

    def handle_server_args(self, server_args) -> None:
        """Fill the tree shape when unset and refuse shapes outside the kernels' limits."""
        steps, top_k, tokens = DEFAULT_TREE_SHAPE
        if getattr(server_args, "speculative_num_steps", None) is None:
            server_args.speculative_num_steps = steps
        if getattr(server_args, "speculative_eagle_topk", None) is None:
            server_args.speculative_eagle_topk = top_k
        if getattr(server_args, "speculative_num_draft_tokens", None) is None:
            server_args.speculative_num_draft_tokens = tokens
        check_shape(self.config.intensity, top_k=server_args.speculative_eagle_topk,
                    depth=server_args.speculative_num_steps, verify=server_args.speculative_num_draft_tokens)

    def req_to_token_extra_len(self, page_size) -> int:
        args = self._server_args()
        return req_to_token_span(args.speculative_eagle_topk, args.speculative_num_steps,
                                 args.speculative_num_draft_tokens, page_size)

    def create_decode_graph_variants(self, info) -> List[dict]:
        """One target-verify graph per verify width the cost model can choose (draft workers: none)."""
        if getattr(info, "is_draft_worker", False):
            return []
        args = self._server_args()
        widths = sorted({w for bs in (1, 8, 64) for w in verify_buckets(bs, self.config.intensity)
                         if w <= args.speculative_num_draft_tokens} | {args.speculative_num_draft_tokens})
        return [{"name": f"eagle4_verify_w{w}", "num_tokens_per_bs": w, "device": getattr(info, "device", None)}
                for w in widths]

    def max_verify_batch_size(self) -> Optional[int]:
        return self.config.max_verify_batch_size

    def create_linear_attn_verify_extension(self, state):
        kind = getattr(state, "kind", "gdn")
        return Mamba2TreeVerify(state) if kind == "mamba2" else GdnTreeVerify(state)

    def _server_args(self):
        from sglang.srt.runtime_context import get_server_args

        return get_server_args()


class GdnTreeVerify(_Extension):
    """GDN layers of the target under tree verify: conv1d and the gated delta rule follow each row's ancestor path
    from the committed state (nothing is written during verify); the accepted path is replayed at commit."""

    def __init__(self, state=None):
        self.state_layout = state
        self.rows = TreeVerifyRows()
        self.records: dict = {}

    def init_cuda_graph_state(self, max_bs, max_num_tokens) -> None:
        # the row tables are derived from the layout tensors inside each captured forward: nothing to preallocate
        self.max_bs, self.max_num_tokens = max_bs, max_num_tokens

    def begin_forward(self, layout, in_graph) -> None:
        self.records.clear()
        if layout is None:
            self.rows.clear()
            return
        self.rows.begin(layout.parent_token, layout.query_start_loc, layout.cache_indices)

    def reads_strided_inputs(self) -> bool:
        return True

    def conv_update(self, layer, mixed_qkv, conv_states, cache_indices, intermediate_conv_window,
                    intermediate_state_indices):
        out = gdn_conv(self.rows, mixed_qkv, conv_states, layer.conv1d.weight.squeeze(1),
                       getattr(layer.conv1d, "bias", None))
        self.records.setdefault(id(layer), {})["x_pre"] = mixed_qkv
        self.records[id(layer)]["conv_states"] = conv_states
        return out

    def recurrent_update(self, layer, query, key, value, a, b, ssm_states, cache_indices, query_start_loc,
                         intermediate_states, intermediate_state_indices):
        shape = GdnShape.of(layer)
        # the three inputs are strided views of one [T, 2 * key + value] conv output
        qkv = torch.as_strided(query, (query.shape[0], shape.gdn_conv_dim), (query.stride(0), 1),
                               query.storage_offset())
        rec = self.records.setdefault(id(layer), {})
        rec.update(qkv=qkv, a=a, b=b, ssm_states=ssm_states, layer=layer, shape=shape)
        return gdn_recurrence(self.rows, qkv, a, b, layer.A_log, layer.dt_bias, ssm_states, shape)

    def commit_state(self, state, state_indices, record_indices, commit_steps, parent) -> bool:
        """Replay the accepted rows (``record_indices`` [bs, steps] verify rows, ``commit_steps`` [bs] path lengths)
        of every recorded layer into its SSM state and conv window (one launch for all layers)."""
        recs = [r for r in self.records.values() if "qkv" in r and "x_pre" in r]
        if not recs:
            return False
        shape = recs[0]["shape"]
        projs = []
        for r in recs:
            cd, vd, hv = shape.gdn_conv_dim, shape.gdn_value_dim, shape.gdn_v_heads
            proj = torch.zeros(r["qkv"].shape[0], cd + vd + 2 * hv, dtype=r["qkv"].dtype, device=r["qkv"].device)
            proj[:, :cd] = r["x_pre"]  # pre-conv inputs (conv windows)
            proj[:, cd + vd: cd + vd + hv] = r["b"]
            proj[:, cd + vd + hv:] = r["a"]
            projs.append(proj)
        ops.gdn_commit_all([r["qkv"] for r in recs], projs, [r["ssm_states"] for r in recs],
                           [r["conv_states"] for r in recs], [r["layer"].A_log for r in recs],
                           [r["layer"].dt_bias for r in recs], state_indices.int(), record_indices.int(),
                           commit_steps.int(), shape)
        return True


class Mamba2TreeVerify(_Extension):
    """Mamba2 layers under tree verify: the tree conv1d (the SSM update follows the same row forest)."""

    def __init__(self, state=None):
        self.state_layout = state
        self.rows = TreeVerifyRows()

    def init_cuda_graph_state(self, max_bs, max_num_tokens) -> None:
        self.max_bs, self.max_num_tokens = max_bs, max_num_tokens

    def begin_forward(self, layout, in_graph) -> None:
        if layout is None:
            self.rows.clear()
        else:
            self.rows.begin(layout.parent_token, layout.query_start_loc, layout.cache_indices)

    def conv_update(self, layer, mixed_qkv, conv_states, cache_indices, intermediate_conv_window,
                    intermediate_state_indices):
        return gdn_conv(self.rows, mixed_qkv, conv_states, layer.conv1d.weight.squeeze(1),
                        getattr(layer.conv1d, "bias", None))


class TreeAttentionVariant:
    """The verify attention SGLang runs for tree rows: this package's paged tree attention (each row sees the
    committed context and its ancestors)."""

    def __init__(self, bs: int, num_tokens: int, head_dim: int):
        self.bs, self.num_tokens, self.head_dim = bs, num_tokens, head_dim

    def run(self, q, k_cache, v_cache, block_table, page, req, ctx_start, ctx_len, extra, n_extra, max_keys=None,
            gate=None):
        return ops.attention(q, k_cache, v_cache, block_table, page, req, ctx_start, ctx_len, extra, n_extra,
                             self.head_dim ** -0.5, max_keys, gate)


class HarnessVerifyInput(_SpecInput):
    def flashinfer_verify_variant(self, bs, num_tokens, q_dtype, kv_dtype, head_dim):
        if q_dtype != torch.bfloat16 or kv_dtype != torch.bfloat16:
            return None  # SGLang's own variant serves other dtypes
        return TreeAttentionVariant(bs, num_tokens, head_dim)


class HarnessWorker(_Worker):
    """The cost-model worker: SGLang prefills and verifies; each decode round drafts a tree sized by the round policy
    and accepts with the fused greedy accept kernel."""

    def create_draft_worker(self, server_args, gpu_id, nccl_port, target_worker):
        return HarnessDraftWorker(server_args, gpu_id, nccl_port, target_worker)

    def init_attention_backends(self) -> None:
        # draft rows attend through this package's tree attention; SGLang's draft backends are not created
        self.draft_attention = "eagle4_b200.tree_attention"

    def _build_trivial_verify_input(self, batch):
        """An idle / root-only round: one verify row per request."""
        bs = len(batch.seq_lens)
        return {"width": 1, "bs": bs, "parent_rows": torch.full((bs, 1), -1, dtype=torch.int32)}

    def forward_batch_generation(self, batch, on_publish=None, grammar_barrier=None, pp_proxy_tensors=None):
        if batch.forward_mode.is_extend() or getattr(batch, "is_extend_in_batch", False):
            return super().forward_batch_generation(batch, on_publish, grammar_barrier, pp_proxy_tensors)
        from sglang.srt.speculative.eagle_worker_common import run_eagle_verify

        spec = self._build_trivial_verify_input(batch) if batch.forward_mode.is_idle() else self.draft(batch)
        batch.spec_info = spec
        return run_eagle_verify(batch=batch, target_worker=self.target_worker,
                                req_to_token_pool=self.req_to_token_pool,
                                token_to_kv_pool_allocator=self.token_to_kv_pool_allocator,
                                plan_stream=None, plan_stream_ctx=None, topk=self.topk,
                                num_draft_tokens=spec["width"], device=self.device, metadata_ready_pre_pad=None,
                                finalize_tree_path=None, grammar_barrier=grammar_barrier,
                                accept_step=self.accept_step)

    def draft(self, batch):  # the draft round of the host's draft worker (tree sized by the round policy)
        return self.draft_worker.draft_round(batch)

    @staticmethod
    def accept_step(verify_input, next_token_ids, draft_tokens, parent_rows):
        """The fused greedy accept over the round's verify rows."""
        return accept_greedy_rows(next_token_ids, draft_tokens, parent_rows)


class HarnessDraftWorker(_DraftWorker):
    """The draft side of SGLang's rounds: this package's draft round (``plugins.host_round.HostDrafter``: draft KV,
    pending rows, draft tree, round policy) over SGLang's requests. SGLang's target worker prefills and verifies;
    ``forward_draft_extend`` takes each prefilled request, ``draft_round`` returns the round's verify rows, and
    ``finish_round`` takes the accepted path (``eagle_harness/sglang/worker.py:532``, ``drafter.py:482``)."""

    drafter = None

    @classmethod
    def for_drafter(cls, drafter) -> "HarnessDraftWorker":
        """A worker around an existing drafter (no SGLang process state)."""
        w = cls.__new__(cls)
        w.drafter = drafter
        return w

    def forward_draft_extend(self, batch, aux_hidden_states, next_token_ids) -> None:
        """After SGLang's prefill of ``batch``: each request's prompt rows (``aux_hidden_states``, the captured target
        layers, rows in batch order) and first token enter the drafter."""
        off = 0
        for req, first in zip(batch.reqs, next_token_ids.tolist()):
            n = len(req.origin_input_ids)
            self.drafter.admit(req.rid, torch.as_tensor(req.origin_input_ids, dtype=torch.int64),
                               aux_hidden_states[off:off + n], first)
            off += n

    def draft_round(self, batch) -> dict:
        """The round's verify input: per request the committed root and the drafted rows chosen by the round policy
        (tokens and parent rows, ``[bs, w]``)."""
        rids = [req.rid for req in batch.reqs]
        tokens, parents = self.drafter.propose(rids)
        return {"width": int(tokens.shape[1]), "bs": len(rids), "rids": rids, "draft_tokens": tokens,
                "parent_rows": parents}

    def finish_round(self, spec: dict, accepted, counts, bonus, aux_hidden_states) -> List[List[int]]:
        """The verify's outcome for ``spec``: the drafter takes the accepted path; returns each request's emitted
        tokens."""
        return self.drafter.accept(spec["rids"], spec["draft_tokens"], accepted, counts, bonus, aux_hidden_states)

    def release(self, rid) -> None:
        self.drafter.release(rid)

    def init_attention_backend(self) -> None:
        self.attention = "eagle4_b200.tree_attention"

    def _capture_cuda_graphs(self) -> None:
        # draft steps are captured per (batch size, step) on first use by the round runner
        self.graphs: dict = {}
