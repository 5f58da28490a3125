"""Shared test setup: import paths, the `gpu` marker, common fixtures."""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "diffusers-cpp_b200")
ORACLE = os.path.join(ROOT, "oracle")
for p in (PKG, ORACLE, ROOT):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


def pytest_collection_modifyitems(config, items):
    import torch

    if torch.cuda.is_available():
        return
    skip = pytest.mark.skip(reason="no CUDA device")
    for it in items:
        if "gpu" in it.keywords:
            it.add_marker(skip)


@pytest.fixture(scope="session")
def ctx():
    import dcpp_b200

    c = dcpp_b200.Context(0)
    yield c
    c.close()


@pytest.fixture(params=[1, 2], ids=["single_sm", "cta_pair"])
def gemm_kind(request, ctx):
    """Run a GEMM test on the single-SM kernel and on the CTA-pair kernel."""
    ctx.set_gemm_kernel(request.param)
    yield request.param
    ctx.set_gemm_kernel(0)


@pytest.fixture(params=[1, 2], ids=["one_tile", "two_tiles"])
def attn_kind(request, ctx):
    """Run an attention test on the one-tile and on the two-tile kernel."""
    ctx.set_attention_kernel(request.param)
    yield request.param
    ctx.set_attention_kernel(0)
