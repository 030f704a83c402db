"""Host logic of orchkv_b200.attention_hook that needs no GPU: the report ids
the collector chooses (against oracle/hook_model.py, the reference hook's
choice, python/orchkv/vllm_integration/attention_hook.py:171-182) and the
check that sends a layer to the fused device reports or to the ordered
device batch.  The fused reports record a block column's heads in order and
the columns in parallel, so they are exact only when no tracker slot is
shared by two columns and no id's low 32 bits equal the no-block marker;
other layers' reports go as one device batch in the hook's order (or, for
the marker, one host call each)."""
import numpy as np
import pytest
import torch

from oracle.hook_model import hook_reports
from orchkv_b200.attention_hook import AttentionScoreCollector

CAP = 1024


def collector(cap=CAP):
    """A collector with only its tracker capacity set (no manager needed)."""
    c = object.__new__(AttentionScoreCollector)
    c._cap = cap
    return c


def ids_in_reference_order(ids):
    h, b = np.nonzero(ids >= 0)           # row-major: head, then block
    return [int(ids[i, j]) for i, j in zip(h, b)]


@pytest.mark.parametrize("mode", ["default", "table", "short_table", "fn", "fn_none"])
def test_block_ids_match_the_reference(mode):
    layer, heads, kv, blk = 3, 5, 150, 16
    nb = (kv + blk - 1) // blk
    aw = torch.rand(2, heads, 1, kv)
    kw = {"default": {},
          "table": {"block_table": torch.tensor([[7 * i - 3 for i in range(nb)]])},
          # a table narrower than the blocks: the rest keep the default ids
          "short_table": {"block_table": torch.tensor([[100 + i for i in range(nb - 4)]])},
          "fn": {"block_id_fn": lambda l, h, bi: 1000 * l + 31 * h + bi},
          "fn_none": {"block_id_fn": lambda l, h, bi: None if (h + bi) % 3 == 0 else h * nb + bi}}[mode]
    ids = collector()._block_ids(layer, heads, nb, kw.get("block_table"), kw.get("block_id_fn"))
    assert ids.shape == (heads, nb)
    want = [bid for bid, _ in hook_reports(layer, aw, blk, kw.get("block_table"),
                                           kw.get("block_id_fn"))]
    assert ids_in_reference_order(ids) == want


def test_device_path_check():
    c = collector()
    heads, nb = 4, 6
    distinct = np.arange(heads * nb, dtype=np.int64).reshape(heads, nb)
    assert c._device_order_ok(distinct)
    # every head of a column shares one id (block-table mode): heads in order
    shared_in_column = np.tile(np.arange(nb, dtype=np.int64) * 5, (heads, 1))
    assert c._device_order_ok(shared_in_column)
    # two columns' ids on one tracker slot: the ordered device batch
    cross = distinct.copy()
    cross[2, 4] = cross[1, 1] + CAP
    assert not c._device_order_ok(cross)
    # the no-block marker in an id's low 32 bits
    marker = distinct.copy()
    marker[0, 0] = 0xFFFFFFFF
    assert not c._device_order_ok(marker)
    # nothing reported, or holes (-1) in the table
    assert c._device_order_ok(np.full((heads, nb), -1, np.int64))
    holes = distinct.copy()
    holes[:, ::2] = -1
    assert c._device_order_ok(holes)
