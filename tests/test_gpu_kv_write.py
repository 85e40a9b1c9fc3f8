"""
GPU parity of the KV writes (reshape_and_cache, copy-on-write block copy):
bit-exact against the reference's golden pools and the oracle.
"""

import os

import numpy as np
import pytest
import torch

from oracle import paged_oracle as O
from tests import cases
from tests.conftest import GOLDEN

pytestmark = pytest.mark.gpu

K = pytest.importorskip("memforge_b200._kernels")


def _bits(t: torch.Tensor) -> np.ndarray:
    if t.dtype == torch.bfloat16:
        return t.cpu().view(torch.int16).numpy().view(np.uint16)
    return t.cpu().numpy()


def _dev_from_storage(arr: np.ndarray, dtype: str) -> torch.Tensor:
    if dtype == "bf16":
        return torch.from_numpy(arr.view(np.int16).copy()).view(torch.bfloat16).cuda()
    return torch.from_numpy(arr.copy()).cuda()


@pytest.mark.parametrize("name", ["scatter_f32_to_f32", "scatter_f32_to_bf16",
                                  "scatter_bf16_to_bf16"])
def test_scatter_kv_matches_reference_golden(name):
    from memforge_b200.paged_gather import scatter_kv
    f = np.load(os.path.join(GOLDEN, name + ".npz"))
    src, pool = name.split("_")[1], name.split("_")[3]
    kp = _dev_from_storage(O.from_f32(f["k0"], pool), pool)
    vp = _dev_from_storage(O.from_f32(f["v0"], pool), pool)
    keys = _dev_from_storage(O.from_f32(f["keys"], src), src)
    values = _dev_from_storage(O.from_f32(f["values"], src), src)
    flat = torch.from_numpy(f["flat"]).cuda()
    scatter_kv(kp, vp, int(f["layer"]), flat, keys, values, int(f["block_size"]))
    torch.cuda.synchronize()
    assert np.array_equal(_bits(kp), f["k_after"])
    assert np.array_equal(_bits(vp), f["v_after"])


@pytest.mark.parametrize("idx_dtype", [torch.int32, torch.int64])
def test_reshape_and_cache_skips_padding_slots(idx_dtype):
    g = torch.Generator(device="cuda").manual_seed(1)
    kp = torch.randn(8, 16, 4, 128, device="cuda", generator=g).bfloat16()
    vp = torch.randn_like(kp)
    before_k, before_v = kp.clone(), vp.clone()
    keys = torch.randn(5, 4, 128, device="cuda", generator=g).bfloat16()
    values = torch.randn_like(keys)
    slots = torch.tensor([3, -1, 40, 127, -1], device="cuda", dtype=idx_dtype)
    K.reshape_and_cache(keys, values, kp, vp, slots)
    torch.cuda.synchronize()
    want_k, want_v = before_k.view(-1, 4, 128).clone(), before_v.view(-1, 4, 128).clone()
    for t, s in enumerate(slots.tolist()):
        if s >= 0:
            want_k[s] = keys[t]
            want_v[s] = values[t]
    assert torch.equal(kp.view(-1, 4, 128), want_k)
    assert torch.equal(vp.view(-1, 4, 128), want_v)


def test_fp32_to_bf16_rounding_is_bit_exact():
    """Ties, NaN, inf and subnormals round exactly like torch's .to(bfloat16)."""
    g = cases.rng(5)
    vals = cases.normal(g, (64, 2, 64), 100.0)
    vals.reshape(-1)[:8] = [np.nan, np.inf, -np.inf, 1.00390625, 1.01171875, 1e-40, -0.0, 3.4e38]
    keys = torch.from_numpy(vals).cuda()
    kp = torch.zeros(4, 16, 2, 64, device="cuda", dtype=torch.bfloat16)
    vp = torch.zeros_like(kp)
    slots = torch.arange(64, device="cuda", dtype=torch.int32)
    K.reshape_and_cache(keys, keys, kp, vp, slots)
    torch.cuda.synchronize()
    got = _bits(kp).reshape(-1)
    nan = np.isnan(vals.reshape(-1))
    # NaN payloads differ between torch's own CPU and GPU casts; only NaN-ness is defined.
    assert np.isnan(O.bf16_to_f32(got[nan])).all()
    assert np.array_equal(got[~nan], O.f32_to_bf16(vals).reshape(-1)[~nan])
    theirs = keys.cpu().to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16).reshape(-1)
    assert np.array_equal(got[~nan], theirs[~nan])


def test_config2_kv_write_bit_exact():
    """BASELINE config 2's write: 64 new tokens at ctx-1 into a 16384-block pool."""
    meta = cases.config2_meta(0)
    NB, H, D = meta["num_blocks"], meta["num_kv_heads"], meta["head_dim"]
    g = torch.Generator(device="cuda").manual_seed(2)
    kp = torch.randn(NB, 16, H, D, device="cuda", generator=g, dtype=torch.bfloat16)
    vp = torch.randn(NB, 16, H, D, device="cuda", generator=g, dtype=torch.bfloat16)
    ref_k, ref_v = kp.clone(), vp.clone()
    B = meta["ctx"].shape[0]
    new_k = torch.randn(B, H, D, device="cuda", generator=g, dtype=torch.bfloat16)
    new_v = torch.randn(B, H, D, device="cuda", generator=g, dtype=torch.bfloat16)
    pos = meta["ctx"].astype(np.int64) - 1
    slots_np = meta["tables"][np.arange(B), pos // 16].astype(np.int64) * 16 + pos % 16
    slots = torch.from_numpy(slots_np.astype(np.int32)).cuda()
    K.reshape_and_cache(new_k, new_v, kp, vp, slots)
    ref_k.view(-1, H, D)[slots.long()] = new_k
    ref_v.view(-1, H, D)[slots.long()] = new_v
    torch.cuda.synchronize()
    assert torch.equal(kp, ref_k) and torch.equal(vp, ref_v)


def test_bad_slot_sets_the_error_word_and_writes_nothing():
    kp = torch.zeros(2, 16, 1, 64, device="cuda", dtype=torch.bfloat16)
    vp = torch.zeros_like(kp)
    keys = torch.ones(2, 1, 64, device="cuda", dtype=torch.bfloat16)
    slots = torch.tensor([5, 32], device="cuda", dtype=torch.int32)   # 32 is past 2*16
    K.reshape_and_cache(keys, keys, kp, vp, slots)
    with pytest.raises(IndexError, match="slot_mapping"):
        K.check_device_errors(kp.device)
    assert float(kp.view(-1, 64)[5].float().sum()) == 64.0
    assert float(kp.float().sum()) == 64.0


def test_copy_blocks_all_layers_bit_exact():
    L_, NB = 3, 10
    kp = torch.randn(L_, NB, 16, 2, 64, device="cuda").bfloat16()
    vp = torch.randn_like(kp)
    ref_k, ref_v = kp.clone(), vp.clone()
    pairs = torch.tensor([[1, 7], [4, 4], [9, 0]], dtype=torch.int32, device="cuda")
    K.copy_blocks(kp, vp, pairs)
    for s, d in [(1, 7), (9, 0)]:
        ref_k[:, d] = ref_k[:, s]
        ref_v[:, d] = ref_v[:, s]
    torch.cuda.synchronize()
    assert torch.equal(kp, ref_k) and torch.equal(vp, ref_v)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32, torch.float16])
@pytest.mark.parametrize("idx_dtype", [torch.int32, torch.int64])
def test_gather_kv_matches_index_select_bit_exact(dtype, idx_dtype):
    """gather_kv / PagedKVPool.gather_flat (paged_gather.py:58-89): (1, H, T, D) copies."""
    from memforge_b200.paged_gather import gather_kv
    L_, NB, H, D = 3, 40, 4, 128
    kp = torch.randn(L_, NB, 16, H, D, device="cuda").to(dtype)
    vp = torch.randn_like(kp)
    g = torch.Generator(device="cuda").manual_seed(5)
    flat = torch.randint(0, NB * 16, (333,), generator=g, device="cuda").to(idx_dtype)
    k, v = gather_kv(kp, vp, 2, flat, 16)
    want_k = kp[2].view(NB * 16, H, D).index_select(0, flat.long()).permute(1, 0, 2)[None]
    want_v = vp[2].view(NB * 16, H, D).index_select(0, flat.long()).permute(1, 0, 2)[None]
    torch.cuda.synchronize()
    assert k.shape == (1, H, 333, D) and k.is_contiguous()
    assert torch.equal(k, want_k) and torch.equal(v, want_v)


def test_gather_kv_odd_head_dim_and_heads_major_layout():
    from memforge_b200 import _kernels as K
    NB, H, D = 12, 3, 40
    cache = torch.randn(NB, H, 16, D, device="cuda")          # standalone operator layout
    flat = torch.tensor([5, 0, 191, 77, 16], device="cuda")
    k, v = K.gather_kv(cache, cache, flat, heads_major=True)
    want = cache.permute(0, 2, 1, 3).reshape(NB * 16, H, D)[flat].permute(1, 0, 2)[None]
    assert torch.equal(k, want) and torch.equal(v, want)


def test_gather_kv_bad_index_reports_and_zero_fills():
    from memforge_b200.paged_gather import gather_kv
    kp = torch.randn(1, 4, 16, 2, 64, device="cuda").bfloat16()
    flat = torch.tensor([3, 64, -2, 7], device="cuda")     # 64 is past 4*16
    k, _ = gather_kv(kp, kp, 0, flat, 16)
    with pytest.raises(IndexError, match="slot_mapping"):
        K.check_device_errors(kp.device)
    assert torch.equal(k[0, :, 0], kp[0].view(64, 2, 64)[3])
    assert float(k[0, :, 1].float().abs().sum()) == 0.0
    assert float(k[0, :, 2].float().abs().sum()) == 0.0


def test_pool_gather_uses_the_kernel_and_matches_the_write():
    """PagedKVPool.write then PagedKVPool.gather returns the rows written (round trip)."""
    from memforge_b200.kv_pool import ModelKVSpec, PagedKVPool
    spec = ModelKVSpec(num_layers=2, num_kv_heads=2, head_dim=64, dtype=torch.bfloat16,
                       device="cuda")
    pool = PagedKVPool(spec, num_blocks=10, block_size=16)
    table = torch.tensor([7, 2, 9], device="cuda")
    phys, slots = pool.slot_indices(table, 5, 40)
    keys = torch.randn(1, 2, 35, 64, device="cuda").bfloat16()
    before = K.launch_counter["gather_kv"]
    pool.write(1, phys, slots, keys, keys * 2)
    k, v = pool.gather(1, phys, slots)
    assert K.launch_counter["gather_kv"] == before + 1
    assert torch.equal(k, keys) and torch.equal(v, keys * 2)
