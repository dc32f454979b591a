"""The committed digests of the configurations' expected results
(tests/golden/config_digests.json, which bench.py checks its pass runs
against) agree with the oracle, on the CPU, for the configurations small
enough to recompute here in seconds; tests/test_gpu_full_configs.py ties
every digest to a driver output checked value by value on the GPU."""
import json
import os

import pytest

HERE = os.path.dirname(os.path.abspath(__file__))


@pytest.mark.parametrize("config", ["config1", "config2"])
def test_digest_matches_the_oracle(config, oracle):
    import make_config_digests as M
    d = json.load(open(os.path.join(HERE, "golden", "config_digests.json")))
    assert M.MAKERS[config]() == d[config]


def test_every_configuration_has_a_digest():
    d = json.load(open(os.path.join(HERE, "golden", "config_digests.json")))
    for k in ["config1", "config2", "config3-i8", "config3-i32", "config3-i64", "config4", "config4b", "config5"]:
        assert len(d[k]) == 64
