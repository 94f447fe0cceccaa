"""Parity on the benchmark configurations at their stated sizes and seeds
(tests/baseline_configs.py): one layer of each model with its whole batch --
the fused append of the step's token (bit-exact pages, and for FP8 pages
bit-exact codes and scales) and the paged decode over ctx + 1 tokens, within
|gpu - ref| <= 2e-3 + 1e-2 * |ref| of the fp64 oracle (the paged decode of
kernels/attention/flash_attention.bm:113-162 generalised to GQA heads)."""
import numpy as np
import pytest

import oracle
from tests import baseline_configs, kvgen
from tests.kvgen import FP8
from tests.test_gpu_kv import check_close, download_pool, make_pool, run_decode

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def dev():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda", 0)


@pytest.mark.parametrize("name", ["C1", "C2", "C4", "C5"])
def test_config_append_and_decode(dev, name):
    c = baseline_configs.build(name)
    pool = make_pool(c, dev)
    got = run_decode(pool, c, 0, dev, fused=True)
    assert pool.check() == 0
    # the oracle's append on the host copy (in place: the arrays are large)
    oracle.kv_append(c.geom, c.data, c.scales, 0, c.k_new[0], c.v_new[0], kvgen.new_token_slots(c))
    gdata, gscales = download_pool(pool, c)
    assert np.array_equal(gdata, c.data), f"{name}: pages after the fused append differ"
    if c.kv == FP8:
        assert np.array_equal(gscales.view(np.uint32), c.scales.view(np.uint32)), f"{name}: scales"
    del gdata, gscales
    ref = oracle.paged_decode_f64(c.geom, c.data, c.scales, 0, c.q[0], c.Hq, c.block_tables,
                                  c.seq_lens, 1.0 / np.sqrt(c.D))
    check_close(got, ref, c.io, name)
    pool.close()
