import os
import sys

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
sys.path.insert(0, HERE)
sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200); runs the product kernels")
    config.addinivalue_line("markers", "slow: full-size model runs (minutes)")


def pytest_collection_modifyitems(config, items):
    # A GPU test that runs past 10 minutes ends the run (stack dump, exit)
    # instead of holding the device.
    for item in items:
        if item.get_closest_marker("gpu") and not item.get_closest_marker("timeout"):
            item.add_marker(pytest.mark.timeout(600, method="thread"))


@pytest.fixture(scope="session")
def oracle():
    import harness
    return harness.Oracle()


@pytest.fixture(scope="session")
def ref():
    import harness
    if not harness.have_ref():
        pytest.skip("reference build oracle/_ref not present")
    return harness.Ref()


@pytest.fixture(scope="session")
def gpu():
    import harness
    import kmap_b200
    kmap_b200.lib()
    if kmap_b200.device_count() < 1:
        pytest.fail("GPU test without a visible CUDA device")
    return harness.Gpu()


@pytest.fixture(scope="session")
def built_lib():
    """libkllm_cuda.so, built if missing (loads without a GPU)."""
    import kmap_b200
    from kmap_b200 import build
    if not os.path.exists(kmap_b200.LIB_PATH):
        build.build()
    return kmap_b200.lib()


TINY_SPECS = {
    # GQA (groups = 2), random norm weights
    "gqa": dict(num_layers=2, hidden_size=128, num_attention_heads=4, num_key_value_heads=2,
                intermediate_size=256, vocab_size=600, max_seq=64, norm_weights="random"),
    # MHA (no REPEAT in the tape), odd-ish sizes
    "mha": dict(num_layers=3, hidden_size=192, num_attention_heads=3, num_key_value_heads=3,
                intermediate_size=320, vocab_size=777, max_seq=96, norm_weights="random",
                seed=5),
    # TinyLlama's head geometry (hd 64, 8 q heads per kv head) at a small width
    "tl": dict(num_layers=2, hidden_size=512, num_attention_heads=8, num_key_value_heads=1,
               intermediate_size=1408, vocab_size=2048, max_seq=160, seed=7),
    # the same with fp16 weights (fp16 value streams) and with 4096-value fp32
    # codebooks (neither bf16 nor fp16: codebook-table streams)
    "tl-fp16": dict(num_layers=2, hidden_size=512, num_attention_heads=8, num_key_value_heads=1,
                    intermediate_size=1408, vocab_size=2048, max_seq=160, seed=7,
                    weight_values="fp16"),
    "tl-pool": dict(num_layers=2, hidden_size=512, num_attention_heads=8, num_key_value_heads=1,
                    intermediate_size=1408, vocab_size=2048, max_seq=160, seed=7,
                    weight_values="pool4096"),
}

#: what the persistent step's weight streams hold for each tiny chip
#: (kllm_infer_stats.stream_values: 0 table slots, 1 bf16, 2 fp16)
TINY_STREAM_VALUES = {"gqa": 1, "mha": 1, "tl": 1, "tl-fp16": 2, "tl-pool": 0}


@pytest.fixture(scope="session")
def chip_dir(tmp_path_factory):
    """Directory holding generated tiny chips (built on first use)."""
    from kmap_b200 import chipgen
    root = tmp_path_factory.mktemp("chips")
    made = {}

    def get(name):
        if name not in made:
            spec = chipgen.ModelSpec(**TINY_SPECS[name])
            made[name] = chipgen.ensure_chip(str(root), spec)
        return made[name]
    return get


@pytest.fixture
def rng():
    return np.random.default_rng(1234)
