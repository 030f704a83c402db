"""The scheduler role of orchkv_b200.vllm_connector on the CPU, against the
reference connector's own run (tests/golden/vllm_connector_scheduler.json,
made by tests/golden/gen_vllm_connector.py from
python/orchkv/vllm_integration/connector.py:227-289,390-421): the same
seeded sequence of prefix-match queries, finished requests, preemptions,
allocation notices and metadata builds gives the same return values and the
same blocks to save and load, in the same order, with the layer count taken
from the extra config or, where it has one, the model config."""
import json
import os

import pytest

from tests.golden.gen_vllm_connector import run
from orchkv_b200.vllm_connector import KVConnectorRole, OrchKvOffloadingConnector

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "vllm_connector_scheduler.json")


@pytest.fixture(scope="module")
def golden():
    with open(GOLDEN) as fh:
        return json.load(fh)


@pytest.mark.parametrize("case", [0, 1])
def test_scheduler_role_matches_reference_run(golden, case):
    c = golden["cases"][case]
    got = run(OrchKvOffloadingConnector, KVConnectorRole.SCHEDULER, c["config"], golden["ops"])
    assert json.loads(json.dumps(got)) == c["results"]
    metas = [r for r in c["results"] if isinstance(r, dict) and r["save"]]
    assert metas and max(len(v) for m in metas for v in m["save"].values()) > 10
