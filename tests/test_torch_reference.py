"""The torch fp32 reference used at full sizes agrees with the numpy oracle (CPU)."""

import numpy as np
import torch

from tests import cases
from tests.gpu_util import torch_reference


def _run(case, window=None):
    q = torch.from_numpy(case.q)
    k = torch.from_numpy(case.k_pool)
    v = torch.from_numpy(case.v_pool)
    tables = torch.from_numpy(case.tables.clip(min=0))
    wk = wv = None
    if window is not None:
        wk = torch.from_numpy(np.concatenate([np.transpose(window[s][1], (1, 0, 2))
                                              for s in range(case.batch)]))
        wv = torch.from_numpy(np.concatenate([np.transpose(window[s][2], (1, 0, 2))
                                              for s in range(case.batch)]))
    return torch_reference(q, k, v, tables, case.ctx_lens, [case.q_per_seq] * case.batch,
                           case.scale, wk, wv).numpy()


def test_decode_matches_oracle():
    c = cases.small_decode_case("t", 11, "f32", 12, 4, 64, [1, 16, 17, 130])
    assert np.allclose(_run(c), cases.oracle_decode(c), atol=1e-5)


def test_multi_row_causal_matches_oracle():
    c = cases.small_decode_case("t", 12, "f32", 10, 2, 64, [5, 40, 77], q_per_seq=5)
    assert np.allclose(_run(c), cases.oracle_decode(c), atol=1e-5)


def test_window_matches_oracle():
    c = cases.small_decode_case("t", 13, "f32", 10, 2, 32, [9, 40], q_per_seq=5)
    g = cases.rng(3)
    window = {s: (int(c.ctx_lens[s]) - 5, cases.normal(g, (2, 5, 32)), cases.normal(g, (2, 5, 32)))
              for s in range(c.batch)}
    assert np.allclose(_run(c, window), cases.oracle_decode(c, window=window), atol=1e-5)
