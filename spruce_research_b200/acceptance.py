"""Whole-model equivalence criteria: how a sparse forward is judged against a reference run.

The reference screens a sparse configuration by comparing the last token's
logits and the final hidden states of the model against a reference run
(benchmarks/all_blocks_equivalence.py:44-50 DEFAULT_ACCEPTANCE, :116-136
tensor_error, :139-156 logits_error, :159-173 passes_acceptance).  The result
keys and the acceptance thresholds are kept as the reference defines them, so
reports from either implementation read the same way.
"""
from __future__ import annotations

import torch

DEFAULT_ACCEPTANCE = {
    "require_finite": True,
    "require_same_top1": True,
    "minimum_top10_overlap": 0.9,
    "minimum_logits_cosine": 0.999,
    "maximum_final_hidden_relative_rmse": 0.02,
}


def tensor_error(actual: torch.Tensor, expected: torch.Tensor) -> dict:
    """Finiteness, max / mean absolute error, RMSE, the expected tensor's RMS and their ratio."""
    if actual.shape != expected.shape:
        raise ValueError(f"shape mismatch: {tuple(actual.shape)} vs {tuple(expected.shape)}")
    a = actual.detach().float()
    e = expected.detach().float().to(a.device)
    diff = a - e
    rmse = diff.square().mean().sqrt().item()
    ref_rms = e.square().mean().sqrt().item()
    return {
        "actual_finite": bool(torch.isfinite(a).all().item()),
        "expected_finite": bool(torch.isfinite(e).all().item()),
        "max_abs": diff.abs().max().item(),
        "mean_abs": diff.abs().mean().item(),
        "rmse": rmse,
        "reference_rms": ref_rms,
        "relative_rmse": rmse / ref_rms if ref_rms else float("inf"),
    }


def logits_error(actual: torch.Tensor, expected: torch.Tensor, top_k: int = 10) -> dict:
    """tensor_error plus cosine similarity and agreement of the top-1 and top-k token ids."""
    out = tensor_error(actual, expected)
    a = actual.detach().float().flatten()
    e = expected.detach().float().flatten().to(a.device)
    a_top = torch.topk(a, k=top_k).indices.tolist()
    e_top = torch.topk(e, k=top_k).indices.tolist()
    out.update({
        "cosine": torch.nn.functional.cosine_similarity(a[None], e[None]).item(),
        "top1_same": a_top[0] == e_top[0],
        "actual_top_ids": a_top,
        "expected_top_ids": e_top,
        "top10_overlap": len(set(a_top) & set(e_top)) / top_k,
    })
    return out


def passes_acceptance(logits: dict, final_hidden: dict, criteria: dict = DEFAULT_ACCEPTANCE) -> bool:
    """True when a run meets every criterion: finite values, same top-1 token, top-10
    overlap, logits cosine and the final hidden states' relative RMSE."""
    finite = all(d[key] for d in (logits, final_hidden) for key in ("actual_finite", "expected_finite"))
    return bool(
        (finite or not criteria["require_finite"])
        and (logits["top1_same"] or not criteria["require_same_top1"])
        and logits["top10_overlap"] >= criteria["minimum_top10_overlap"]
        and logits["cosine"] >= criteria["minimum_logits_cosine"]
        and final_hidden["relative_rmse"] <= criteria["maximum_final_hidden_relative_rmse"]
    )
