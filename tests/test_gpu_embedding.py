"""GPU parity: token embedding gather (bitwise, both layouts) and the id
validation of the host-ids entry point."""

import ctypes

import numpy as np
import pytest
import torch

from gpu_util import P, S, call, dev, empty, host
from helpers import assert_bitwise, splitmix_normal
import tfx
from tfx import _lib

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("layout,hidden,vocab,length", [
    (0, 768, 5000, 300), (1, 768, 5000, 300), (0, 6, 50, 17), (1, 6, 50, 17), (1, 1024, 7, 1000)])
def test_embedding_matches_oracle(orc, layout, hidden, vocab, length):
    table = splitmix_normal(hidden * vocab, 0x7E4F0C00 + layout + hidden)
    ids = np.random.default_rng(hidden + layout).integers(0, vocab, length).astype(np.int64)
    td = dev(table)
    out = empty(hidden * length)
    call("tfx_embedding_f32", P(td), ids.ctypes.data_as(ctypes.c_void_p), P(out), hidden, vocab,
         length, layout, S())
    want = orc.embedding_f32(table, ids, hidden, vocab, layout)
    assert_bitwise(host(out), want, f"embedding layout {layout}")
    # device ids give the same result
    idd = torch.from_numpy(ids).cuda()
    out2 = empty(hidden * length)
    call("tfx_embedding_gather_f32", P(td), P(idd), P(out2), hidden, vocab, length, layout, S())
    assert_bitwise(host(out2), want, f"embedding gather layout {layout}")


def test_embedding_rejects_ids_outside_vocabulary():
    hidden, vocab = 8, 10
    td = dev(np.ones(hidden * vocab, np.float32))
    out = empty(hidden * 3)
    ids = np.array([1, 10, 2], np.int64)
    rc = _lib.lib.tfx_embedding_f32(P(td), ids.ctypes.data_as(ctypes.c_void_p), P(out), hidden,
                                    vocab, 3, 1, S())
    assert rc == -1 and b"position 1" in _lib.lib.tfx_last_error_string()
    # device ids out of range produce NaN vectors, the other tokens are gathered
    idd = torch.from_numpy(ids).cuda()
    call("tfx_embedding_gather_f32", P(td), P(idd), P(out), hidden, vocab, 3, 1, S())
    got = host(out).reshape(3, hidden)
    assert np.all(np.isnan(got[1])) and np.all(got[0] == 1.0) and np.all(got[2] == 1.0)
