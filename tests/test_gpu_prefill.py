"""
GPU parity of varlen chunked prefill (the tcgen05 prefill kernel, and its
split with the decode kernel inside one call) against the numpy oracle.
Tolerance: 2e-2 abs + 1e-2 rel for bf16/fp16.
"""

import math

import numpy as np
import pytest
import torch

from oracle.paged_oracle import varlen_attention
from tests import cases
from tests.gpu_util import assert_close, to_dev, to_np32

pytestmark = pytest.mark.gpu

K = pytest.importorskip("memforge_b200._kernels")


def varlen_case(seed, dtype, hq, hkv, D, runs, kv_std=1.0, q_std=1.0):
    """runs: list of (q_len, kv_len): rows are positions kv_len-q_len .. kv_len-1."""
    g = cases.rng(seed)
    kv = [k for _, k in runs]
    need = sum((k + 15) // 16 for k in kv)
    NB = need + 16
    tables = cases.disjoint_tables(g, kv, NB)
    total = sum(q for q, _ in runs)
    rnd = (lambda x: cases.bf16_round(x)) if dtype == "bf16" else (
        (lambda x: x.astype(np.float16).astype(np.float32)) if dtype == "f16" else (lambda x: x))
    q = rnd(cases.normal(g, (total, hq, D), q_std))
    kp = rnd(cases.normal(g, (NB, 16, hkv, D), kv_std))
    vp = rnd(cases.normal(g, (NB, 16, hkv, D), kv_std))
    cu = np.zeros(len(runs) + 1, np.int32)
    cu[1:] = np.cumsum([q for q, _ in runs])
    return dict(q=q, kp=kp, vp=vp, tables=tables, cu=cu, kv=np.array(kv, np.int32),
                runs=runs, dtype=dtype, scale=1 / math.sqrt(D), hkv=hkv)


def run_gpu(c):
    dt = c["dtype"]
    q = to_dev(c["q"], dt)
    out = torch.empty_like(q)
    K.paged_attention(q, out, to_dev(c["kp"], dt), to_dev(c["vp"], dt),
                      torch.from_numpy(c["tables"].clip(min=0)).cuda(),
                      torch.from_numpy(c["kv"]).cuda(),
                      cu_seqlens_q=torch.from_numpy(c["cu"]).cuda(),
                      max_q_len=max(ql for ql, _ in c["runs"]), scale=c["scale"], causal=True)
    torch.cuda.synchronize()
    K.check_device_errors(q.device)
    return to_np32(out)


def run_oracle(c):
    seq_ids, positions = [], []
    for s, (ql, kl) in enumerate(c["runs"]):
        for i in range(ql):
            seq_ids.append(s)
            positions.append(kl - ql + i)
    tables = [t[t >= 0] for t in c["tables"]]
    out = varlen_attention(np.transpose(c["q"], (1, 0, 2)), c["kp"][None], c["vp"][None], 0,
                           tables, seq_ids, positions, 16, scale=c["scale"])
    return np.transpose(out, (1, 0, 2))


def check(c, what=""):
    assert_close(run_gpu(c), run_oracle(c), c["dtype"], what)


@pytest.mark.parametrize("q_len", [3, 32, 33, 100, 128, 257, 600])
def test_full_prompt(q_len):
    check(varlen_case(1, "bf16", 32, 8, 128, [(q_len, q_len)]), f"prompt {q_len}")


@pytest.mark.parametrize("prefix,chunk", [(16, 512), (700, 512), (1024, 300), (5, 129), (0, 512)])
def test_chunk_over_a_paged_prefix(prefix, chunk):
    check(varlen_case(2, "bf16", 32, 8, 128, [(chunk, prefix + chunk)]), f"{prefix}+{chunk}")


def test_several_prefill_sequences():
    runs = [(512, 512 + 300), (200, 200), (64, 64 + 1500), (1, 900), (37, 40)]
    check(varlen_case(3, "bf16", 32, 8, 128, runs), "multi")


def test_prefill_mixed_with_decodes_in_one_call():
    """BASELINE config 3's shape in miniature: chunks beside single decode tokens."""
    g = cases.rng(4)
    runs = [(int(l), int(l + p)) for l, p in zip(g.integers(20, 300, 4), g.integers(0, 400, 4))]
    runs += [(1, int(c)) for c in g.integers(16, 800, 12)]
    order = g.permutation(len(runs))
    runs = [runs[i] for i in order]
    check(varlen_case(5, "bf16", 32, 8, 128, runs), "mixed")


@pytest.mark.parametrize("hq,hkv", [(8, 8), (16, 8), (64, 8), (8, 1), (40, 8), (48, 8), (56, 8),
                                     (64, 4)])
def test_gqa_groups(hq, hkv):
    check(varlen_case(6, "bf16", hq, hkv, 128, [(150, 400), (77, 77)]), f"gqa {hq}/{hkv}")


def test_many_sequences_in_the_sorted_work_list():
    """300 short runs of varied length: the kernel sorts its work list by kv_len
    (longest first) across more sequences than it has threads."""
    g = np.random.default_rng(8)
    runs = [(int(q), int(q + g.integers(0, 300))) for q in g.integers(3, 40, size=300)]
    check(varlen_case(8, "bf16", 32, 8, 128, runs), "300 runs")


def test_fp16():
    check(varlen_case(7, "f16", 32, 8, 128, [(300, 500)]), "fp16")


def test_growing_scores_trigger_rescales():
    """Later keys score higher and higher: the lazy O correction must fire."""
    c = varlen_case(8, "bf16", 16, 4, 128, [(256, 1024)])
    ramp = np.linspace(0.2, 6.0, c["kp"].shape[0] * 16, dtype=np.float32).reshape(-1, 16, 1, 1)
    # scale K so that block order in the table increases the score magnitude
    order = np.argsort(c["tables"][0][c["tables"][0] >= 0])
    kp = c["kp"].copy()
    t = c["tables"][0]
    for L, blk in enumerate(t[t >= 0]):
        kp[blk] *= 1.0 + 0.05 * L
    c["kp"] = cases.bf16_round(kp)
    c["q"] = cases.bf16_round(c["q"] * 3.0)
    check(c, "rescale")


def test_unwritten_slots_of_the_last_page_are_ignored():
    c = varlen_case(9, "bf16", 32, 8, 128, [(100, 250)])
    a = run_gpu(c)
    last = c["tables"][0][(250 - 1) // 16]
    c["kp"][last, 250 % 16:] = np.nan
    c["vp"][last, 250 % 16:] = np.nan
    b = run_gpu(c)
    assert np.isfinite(b).all()
    assert np.array_equal(a, b)


def test_config3_pass_shape():
    """One pass of BASELINE config 3 (16 chunks of <= 512 tokens + 48 decodes)."""
    meta = cases.config3_meta(0)
    ql, kl = cases.config3_pass(meta, 0)
    runs = list(zip(ql.tolist(), kl.tolist()))
    c = varlen_case(10, "bf16", 32, 8, 128, runs)
    got = run_gpu(c)
    want = run_oracle(c)
    assert_close(got, want, "bf16", "config3")
