"""The reference's vLLM attention-hook reports, restated.

TEST INFRASTRUCTURE ONLY: the sequence of tm_report_attn calls the
reference's AttentionScoreCollector.collect makes for one layer
(python/orchkv/vllm_integration/attention_hook.py:105-189): scores are the
mean over batch, query positions and the block's token positions of the
weights zero-padded to whole blocks (:118-140), reported head by head, block
by block, to block_id_fn(layer, head, block) if given, else
block_table[0, block] where the table is wide enough, else
layer * heads * n_blocks + head * n_blocks + block, skipping None and
negative ids (:155-189).  The scores come from torch's own mean over the
padded view, as in the reference.
"""
from __future__ import annotations

import torch


def block_means(aw: torch.Tensor, block_size: int) -> torch.Tensor:
    """[batch, heads, q_len, kv_len] -> [heads, n_blocks] (weights' dtype)."""
    bs, h, q, kv = aw.shape
    nb = (kv + block_size - 1) // block_size
    pad = nb * block_size - kv
    if pad:
        aw = torch.nn.functional.pad(aw, (0, pad))
    return aw.view(bs, h, q, nb, block_size).mean(dim=(0, 2, 4))


def hook_reports(layer: int, aw: torch.Tensor, block_size: int, block_table=None,
                 block_id_fn=None):
    """[(block id, score as float)] in the order the reference reports them."""
    heads = aw.shape[1]
    scores = block_means(aw, block_size).float().cpu()
    nb = scores.shape[1]
    out = []
    for h in range(heads):
        for bi in range(nb):
            if block_id_fn is not None:
                bid = block_id_fn(layer, h, bi)
            elif block_table is not None and bi < block_table.shape[-1]:
                bid = int(block_table[0, bi])
            else:
                bid = layer * heads * nb + h * nb + bi
            if bid is not None and bid >= 0:
                out.append((int(bid), float(scores[h, bi])))
    return out
