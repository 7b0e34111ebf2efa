"""FlatGate on the GPU: the reference's module and checkpoint format, CUDA scoring.

Mirrors selector/gate.py:16-175 of the reference: per-layer ``Wq, Wk`` of
shape ``[L, d, p]`` (kaiming-uniform init, a = sqrt(5)), ``forward(q_feat,
k_feat) -> [L, G, qb, kb]`` raw MaxSim scores divided by sqrt(p).  Scores come
from the fixed-order fp32 kernels of csrc/select.cu: one dot per block pair
for P = 1, the max over the P x P prototype pairs for P > 1 (up to 8), and
``score_projected_candidates`` scores per-row candidate nodes the same way.
``select_blocks`` adds the fused top-k + packing that produces
``selected_blocks`` rows without materialising the score matrix (P = 1).
"""
from __future__ import annotations

import math

import torch
import torch.nn as nn

from .. import native


class FlatGate(nn.Module):
    def __init__(self, num_layers, head_dim, proj_dim=None):
        super().__init__()
        d = head_dim
        p = proj_dim or head_dim
        self.proj_dim = p
        self.Wq = nn.Parameter(torch.empty(num_layers, d, p))
        self.Wk = nn.Parameter(torch.empty(num_layers, d, p))
        for W in (self.Wq, self.Wk):
            nn.init.kaiming_uniform_(W, a=math.sqrt(5))

    @staticmethod
    def _check_prototypes(feat: torch.Tensor, single: bool = True) -> None:
        if feat.dim() != 5:
            raise ValueError(f"features must be [L, G, blocks, P, d], got {tuple(feat.shape)}")
        if single and feat.shape[3] != 1:
            raise ValueError("the fused top-k selector scores one prototype per block (P = 1)")
        if not 1 <= feat.shape[3] <= 8:
            raise ValueError(f"the B200 MaxSim gate takes 1 to 8 prototypes, got P = {feat.shape[3]}")

    @torch.no_grad()
    def project_queries(self, q_feat):
        """``[L, G, qb, P, d] -> [L, G, qb, P, p]`` fp32 (selector/gate.py:120-122)."""
        return torch.stack([native.gate_project(q_feat[l], self.Wq[l]) for l in range(q_feat.shape[0])])

    @torch.no_grad()
    def project_keys(self, k_feat):
        """``[L, G, nodes, P, d] -> [L, G, nodes, P, p]`` fp32 (:124-127)."""
        return torch.stack([native.gate_project(k_feat[l], self.Wk[l]) for l in range(k_feat.shape[0])])

    @torch.no_grad()
    def forward(self, q_feat, k_feat):
        """``q_feat [L, G, qb, P, d]``, ``k_feat [L, G, kb, P, d]`` -> MaxSim scores ``[L, G, qb, kb]`` (:80-101)."""
        self._check_prototypes(q_feat, single=False)
        self._check_prototypes(k_feat, single=False)
        L, G, qb, P = q_feat.shape[:4]
        kb = k_feat.shape[2]
        if k_feat.shape[3] != P:
            raise ValueError("query and key features must have the same number of prototypes")
        if P == 1:
            qp = self.project_queries(q_feat)[:, :, :, 0]
            kp = self.project_keys(k_feat)[:, :, :, 0]
            s = native.gate_scores(qp.reshape(L * G, qb, -1), kp.reshape(L * G, kb, -1))
            return s.view(L, G, qb, kb)
        qp = self.project_queries(q_feat)
        kp = self.project_keys(k_feat)
        s = native.gate_maxsim(qp.reshape(L * G, qb, P, -1), kp.reshape(L * G, kb, P, -1))
        return s.view(L, G, qb, kb)

    @torch.no_grad()
    def score_projected_candidates(self, projected_q, projected_k, candidate_ids, layer_chunk=1):
        """Scores of per-row candidate nodes (:132-171): projected_q ``[L, G, qb, P, p]``,
        projected_k ``[L, G, nodes, P, p]``, candidate_ids ``[L, G, qb, C]`` -> ``[L, G, qb, C]``."""
        if projected_q.dim() != 5 or projected_k.dim() != 5 or candidate_ids.dim() != 4:
            raise ValueError("candidate scoring expects q/k 5-D and IDs 4-D")
        L, G, qb = projected_q.shape[:3]
        if projected_k.shape[:2] != (L, G) or candidate_ids.shape[:3] != (L, G, qb):
            raise ValueError("candidate scoring layer/group/query dimensions mismatch")
        if layer_chunk < 1:
            raise ValueError("layer_chunk must be >= 1")
        nodes, P, p = projected_k.shape[2:]
        C = candidate_ids.shape[-1]
        s = native.gate_maxsim(projected_q.reshape(L * G, qb, P, p).float(),
                               projected_k.reshape(L * G, nodes, P, p).float(),
                               candidate_ids.reshape(L * G, qb, C))
        return s.view(L, G, qb, C)

    @torch.no_grad()
    def score_candidates(self, q_feat, k_feat, candidate_ids):
        """Project Q/K once, then score the candidates (:173-175)."""
        return self.score_projected_candidates(self.project_queries(q_feat), self.project_keys(k_feat),
                                               candidate_ids)

    @torch.no_grad()
    def select_blocks(self, q_feat, k_feat, k_selected, local_window=0, sink_blocks=1, out=None):
        """Flat top-k routes for every layer: int32 ``[1, L, G, qb, K]``.

        Equivalent to masking future / sink / local blocks, ``topk(K - forced)``
        and ``selected_ids_to_blocks(ids, K, local_window, key_blocks=qb,
        sink_blocks)`` (scripts/route_overrides.py:187-205,
        scripts/export_selected_blocks.py:80-175), with ties to the lowest id.
        """
        self._check_prototypes(q_feat)
        L, G, qb = q_feat.shape[:3]
        if out is None:
            out = torch.empty((1, L, G, qb, k_selected), device=q_feat.device, dtype=torch.int32)
        qp = self.project_queries(q_feat)[:, :, :, 0]
        kp = self.project_keys(k_feat)[:, :, :, 0]
        for l in range(L):
            native.gate_select(qp[l][None], kp[l][None], k_selected, local_window, sink_blocks, out=out[:, l])
        return out


def load_gate(path, device):
    """Load a gate checkpoint ``{state_dict, config}`` (scripts/eval_tree_traversal.py:26-32)."""
    ck = torch.load(path, map_location="cpu", weights_only=True)  # plain tensors and a config dict
    cfg = ck["config"]
    gate = FlatGate(cfg["num_layers"], cfg["head_dim"], cfg["proj_dim"])
    gate.load_state_dict(ck["state_dict"])
    return gate.to(device).eval(), cfg
