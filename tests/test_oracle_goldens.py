"""The oracle reproduces the committed golden outputs (tests/golden/config_goldens.npz)
from the regenerated inputs, whose SHA-256 must match the one the outputs were made from."""
import json
import os

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
GOLD = np.load(os.path.join(HERE, "golden", "config_goldens.npz"))
META = json.loads(bytes(GOLD["meta_json"]).decode())

import sys  # noqa: E402
sys.path.insert(0, HERE)
from golden import make_config_goldens as MG  # noqa: E402


@pytest.mark.parametrize("index", range(len(MG.SPECS)), ids=[s[0] for s in MG.SPECS])
def test_golden_inputs_and_oracle(oracle, index):
    inp = MG.spec_inputs(index)
    meta = META[index]
    assert meta["name"] == inp["name"]
    assert inp["sha256"] == meta["sha256"], "input generator changed: regenerate the goldens"
    name = inp["name"]
    hl = inp["hist_len"]
    ids, traces, st = oracle.sample_rows(inp["logits"], inp["vocab"], inp["softcap"],
                                         inp["history"] if hl else None, inp["history_len"] if hl else None,
                                         inp["mask_table"], inp["mask_state"], inp["params"],
                                         rng_state=GOLD[f"{name}/rng_state"], threads=os.cpu_count() or 1)
    assert ids.tolist() == GOLD[f"{name}/ids"].tolist()
    assert st.tolist() == GOLD[f"{name}/rng_state_after"].tolist()
