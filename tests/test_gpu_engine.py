"""
The kernels serving a real model: a tiny randomly initialised Llama (no
weights are downloaded) run through ``memforge_b200.paged_cache.PagedCache``,
the ``memforge_paged`` attention function and the graphed decoder, against
the same model on transformers' own ``DynamicCache`` + sdpa path.

Follows the reference's end-to-end checks: logits of a prefill plus decode
steps equal to ``DynamicCache``'s (``tests/python/test_paged_cache.py:23-54``),
and graphed decode tokens identical to the eager paged path
(``tests/python/test_graphed_paged_decode.py:41-44``).

* fp32, head_dim 64: the cache's KV write and gather kernels feed sdpa, so the
  logits must be bitwise equal to ``DynamicCache``'s, as in the reference test;
  with the paged attention kernel reading the pool (lazy mode) they must agree
  within 1e-4.
* bf16, head_dim 128: the tcgen05 prefill kernel serves the prompt and the
  decode kernel the steps; logits agree with the bf16 sdpa path within bf16
  noise and the greedy tokens match.
"""

import pytest
import torch

pytestmark = pytest.mark.gpu

transformers = pytest.importorskip("transformers")

from memforge_b200 import attention_backend as AB  # noqa: E402
from memforge_b200.kv_pool import ModelKVSpec, PagedKVPool  # noqa: E402
from memforge_b200.paged_cache import PagedCache  # noqa: E402

VOCAB = 256


def tiny_llama(head_dim, dtype, layers=2, seed=0):
    from transformers import LlamaConfig, LlamaForCausalLM
    torch.manual_seed(seed)
    heads, kv_heads = 4, 2
    cfg = LlamaConfig(vocab_size=VOCAB, hidden_size=heads * head_dim, intermediate_size=256,
                      num_hidden_layers=layers, num_attention_heads=heads,
                      num_key_value_heads=kv_heads, head_dim=head_dim,
                      max_position_embeddings=4096, eos_token_id=1, bos_token_id=0,
                      pad_token_id=0, attn_implementation="sdpa")
    return LlamaForCausalLM(cfg).to(device="cuda", dtype=dtype).eval()


def make_pool(model, dtype, blocks=64):
    spec = ModelKVSpec.from_config(model.config, dtype, "cuda")
    return PagedKVPool(spec, num_blocks=blocks, block_size=16)


PROMPT = [5, 17, 33, 2, 90, 41, 7, 7, 250, 3, 19, 64, 128, 77, 12, 200, 9, 31, 44, 101,
          6, 8, 150, 11, 99, 23, 57, 14, 3, 88, 60, 2, 200, 45, 33]
TABLE = [9, 3, 17, 1, 25, 8, 40, 33]   # scattered, out of order


def dynamic_run(model, steps):
    from transformers.cache_utils import DynamicCache
    cache = DynamicCache()
    ids = torch.tensor([PROMPT], device="cuda")
    logits = []
    with torch.no_grad():
        out = model(input_ids=ids, past_key_values=cache, use_cache=True)
        logits.append(out.logits)
        tok = int(out.logits[0, -1].argmax())
        for _ in range(steps):
            out = model(input_ids=torch.tensor([[tok]], device="cuda"), past_key_values=cache,
                        use_cache=True)
            logits.append(out.logits)
            tok = int(out.logits[0, -1].argmax())
    return logits


def paged_run(model, pool, steps, lazy, tokens_from=None):
    """Prefill + greedy decode through PagedCache; lazy: the paged kernel reads the pool."""
    cache = PagedCache(pool, TABLE, lazy_read=lazy)
    ids = torch.tensor([PROMPT], device="cuda")
    logits, used = [], 0

    def fwd(x):
        nonlocal used
        cache.begin_step(TABLE)
        with torch.no_grad():
            if lazy:
                with AB.backend_enabled_on(model), AB.paged_attention_context(pool, cache) as b:
                    out = model(input_ids=x, past_key_values=cache, use_cache=True)
                used += b.used
                return out
            return model(input_ids=x, past_key_values=cache, use_cache=True)
    out = fwd(ids)
    logits.append(out.logits)
    tok = int(out.logits[0, -1].argmax())
    for i in range(steps):
        if tokens_from is not None:
            tok = int(tokens_from[i][0, -1].argmax())
        out = fwd(torch.tensor([[tok]], device="cuda"))
        logits.append(out.logits)
        tok = int(out.logits[0, -1].argmax())
    return logits, used, cache


def test_paged_cache_matches_dynamic_cache_exactly_fp32():
    model = tiny_llama(64, torch.float32)
    want = dynamic_run(model, 6)
    got, _, cache = paged_run(model, make_pool(model, torch.float32), 6, lazy=False)
    for a, b in zip(want, got):
        assert torch.equal(a, b)
    assert cache.position == len(PROMPT) + 6


def test_paged_kernel_reading_the_pool_matches_dynamic_cache_fp32():
    model = tiny_llama(64, torch.float32)
    want = dynamic_run(model, 6)
    got, used, cache = paged_run(model, make_pool(model, torch.float32), 6, lazy=True)
    assert used == 7 * model.config.num_hidden_layers   # every layer of every pass
    for a, b in zip(want, got):
        assert torch.allclose(a, b, atol=1e-4, rtol=1e-4), float((a - b).abs().max())
    assert [int(x[0, -1].argmax()) for x in want] == [int(x[0, -1].argmax()) for x in got]


def test_bf16_head_dim_128_prefill_and_decode_kernels():
    model = tiny_llama(128, torch.bfloat16)
    want = dynamic_run(model, 6)
    got, used, _ = paged_run(model, make_pool(model, torch.bfloat16), 6, lazy=True,
                             tokens_from=want)
    assert used == 7 * model.config.num_hidden_layers
    for a, b in zip(want, got):
        a, b = a.float(), b.float()
        err = (a - b).abs().max()
        assert float(err) <= 5e-2 + 2e-2 * float(a.abs().max()), float(err)


def test_prefix_seeded_chunk_reads_the_shared_prefix_from_the_pool():
    """seed_position: the second half of the prompt runs as a chunk over the first."""
    model = tiny_llama(64, torch.float32)
    pool = make_pool(model, torch.float32)
    full = PagedCache(pool, TABLE, lazy_read=True)
    half = len(PROMPT) // 2
    with torch.no_grad(), AB.backend_enabled_on(model):
        full.begin_step(TABLE)
        with AB.paged_attention_context(pool, full):
            whole = model(input_ids=torch.tensor([PROMPT], device="cuda"),
                          past_key_values=full, use_cache=True).logits
        part = PagedCache(pool, TABLE, lazy_read=True)
        part.seed_position(half)
        part.begin_step(TABLE)
        with AB.paged_attention_context(pool, part):
            tail = model(input_ids=torch.tensor([PROMPT[half:]], device="cuda"),
                         position_ids=torch.arange(half, len(PROMPT), device="cuda")[None],
                         past_key_values=part, use_cache=True).logits
    assert torch.allclose(whole[:, half:], tail, atol=1e-4, rtol=1e-4)


def test_rollback_moves_the_cursor_only():
    model = tiny_llama(64, torch.float32)
    pool = make_pool(model, torch.float32)
    _, _, cache = paged_run(model, pool, 3, lazy=True)
    before = pool.key_pool.clone()
    cache.rollback(2)
    assert cache.position == len(PROMPT) + 1
    assert torch.equal(pool.key_pool, before)


def test_graphed_decode_tokens_identical_to_eager_paged():
    from memforge_b200.graphed_decode import GraphedPagedDecoder
    model = tiny_llama(64, torch.float32)
    prompts = [PROMPT, PROMPT[:9], PROMPT[3:30]]
    tables = [[9, 3, 17, 1], [25, 8, 40, 33], [2, 4, 6, 10]]
    steps = 12
    # eager paged reference: each sequence alone, PagedCache + memforge_paged
    pool_a = make_pool(model, torch.float32)
    want = []
    for p, t in zip(prompts, tables):
        cache = PagedCache(pool_a, t, lazy_read=True)
        toks = []
        with torch.no_grad(), AB.backend_enabled_on(model):
            cache.begin_step(t)
            with AB.paged_attention_context(pool_a, cache):
                out = model(input_ids=torch.tensor([p], device="cuda"), past_key_values=cache,
                            use_cache=True)
            tok = int(out.logits[0, -1].argmax())
            for _ in range(steps):
                toks.append(tok)
                cache.begin_step(t)
                with AB.paged_attention_context(pool_a, cache):
                    out = model(input_ids=torch.tensor([[tok]], device="cuda"),
                                past_key_values=cache, use_cache=True)
                tok = int(out.logits[0, -1].argmax())
        want.append(toks)
    # graphed: the same prefills, then all three sequences decoded together
    pool_b = make_pool(model, torch.float32)
    first, ctx = [], []
    for p, t in zip(prompts, tables):
        cache = PagedCache(pool_b, t, lazy_read=True)
        with torch.no_grad(), AB.backend_enabled_on(model):
            cache.begin_step(t)
            with AB.paged_attention_context(pool_b, cache):
                out = model(input_ids=torch.tensor([p], device="cuda"), past_key_values=cache,
                            use_cache=True)
        first.append(int(out.logits[0, -1].argmax()))
        ctx.append(len(p))
    before = model.config._attn_implementation
    dec = GraphedPagedDecoder(model, pool_b, max_batch=4, max_model_len=64)
    got = [[] for _ in prompts]
    toks = first
    ttabs = [torch.tensor(t, device="cuda") for t in tables]
    for _ in range(steps):
        for i, tk in enumerate(toks):
            got[i].append(tk)
        logits = dec.step(toks, ctx, ttabs)
        toks = [int(x) for x in logits.argmax(-1)]
        ctx = [c + 1 for c in ctx]
    assert got == want
    assert dec.replays == steps and dec.captures == 1
    assert model.config._attn_implementation == before


def test_unbound_calls_run_the_kernel_over_the_handed_keys():
    """No binding: a plain prefill with memforge_paged enabled equals sdpa."""
    model = tiny_llama(64, torch.float32)
    ids = torch.tensor([PROMPT, PROMPT[::-1]], device="cuda")
    with torch.no_grad():
        want = model(input_ids=ids, use_cache=False).logits
        with AB.backend_enabled_on(model):
            got = model(input_ids=ids, use_cache=False).logits
    assert torch.allclose(want, got, atol=1e-4, rtol=1e-4)


def test_unbound_padded_batch_is_rejected():
    model = tiny_llama(64, torch.float32)
    ids = torch.tensor([PROMPT[:8], PROMPT[:8]], device="cuda")
    mask = torch.ones_like(ids)
    mask[1, :3] = 0
    with torch.no_grad(), AB.backend_enabled_on(model):
        with pytest.raises(NotImplementedError):
            model(input_ids=ids, attention_mask=mask, use_cache=False)
