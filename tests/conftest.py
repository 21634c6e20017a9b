import os
import sys

import pytest

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (run with -m gpu on a B200)")


def pytest_collection_modifyitems(config, items):
    import torch
    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for item in items:
        if "gpu" in item.keywords:
            item.add_marker(skip)


@pytest.fixture(scope="session")
def tiny_corpus(tmp_path_factory):
    from modded_nanogpt_b200.data.shards import write_synthetic_corpus
    root = tmp_path_factory.mktemp("corpus")
    write_synthetic_corpus(root, train_tokens=300_000, val_tokens=40_000, shard_tokens=200_000,
                           doc_len="geometric", mean_len=200.0)
    return str(root)
