"""Shared fixtures. Tests marked `gpu` need a B200; everything else runs on CPU.

The seeded synthetic model (the reference's SD-card format) is generated once
per session by libqwen_b200's generator; its SHA-256 digests are pinned by the
golden fixtures made from the reference's own model_backend.py.
"""
import json
import os
import sys
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parents[1]
PKG = REPO / 'fpga2026-40999-llm-accelerator-for-qwen2.5-0.5b-on-fpga_b200'
for p in (str(PKG), str(REPO)):
    if p not in sys.path:
        sys.path.insert(0, p)

GOLDEN_SEED = 2026


def pytest_configure(config):
    config.addinivalue_line('markers', 'gpu: needs a B200 (run with -m gpu)')


@pytest.fixture(scope='session')
def golden():
    g = json.loads((REPO / 'tests/golden' / f'qwen_seed{GOLDEN_SEED}.json').read_text())
    import numpy as np
    g['arrays'] = dict(np.load(REPO / 'tests/golden' / f'qwen_seed{GOLDEN_SEED}.npz'))
    return g


@pytest.fixture(scope='session')
def sd_root(tmp_path_factory):
    """Folder holding QWEN25/* for the golden seed (about 0.77 GB)."""
    import qwen_b200
    from qwen_b200 import _lib
    _lib.lib()
    root = tmp_path_factory.mktemp('sd')
    assert qwen_b200.lib().qwen_b200_synth_write(str(root).encode(), GOLDEN_SEED) == 0
    return root


@pytest.fixture(scope='session')
def oracle_model(sd_root):
    from oracle.ref import RefModel
    m = RefModel(sd_root, capacity=512, threads=os.cpu_count() or 1)
    yield m
    m.close()
