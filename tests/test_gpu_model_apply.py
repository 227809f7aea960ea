"""``*ModelWithHead.apply`` (the reference's model call without a cache) on the GPU kernels against the
oracle: all-position logits, the last-n slice, and a right-padded mask."""
import pytest
import torch

from jaxml_b200 import GemmaModelWithHead, GPTNeoXModelWithHead, LlamaModelWithHead
from oracle import jaxml_oracle as O

pytestmark = pytest.mark.gpu

CLASSES = {"llama": LlamaModelWithHead, "neox": GPTNeoXModelWithHead, "gemma3": GemmaModelWithHead}


def _close(got, want, dtype):
    got, want = got.float().cpu(), want.float().cpu()
    if dtype == torch.float32:
        assert torch.allclose(got, want, rtol=1e-4, atol=1e-5), (got - want).abs().max().item()
    else:
        assert (got - want).abs().max().item() <= 2e-2, (got - want).abs().max().item()


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16], ids=["f32", "bf16"])
@pytest.mark.parametrize("family", ["llama", "neox", "gemma3"])
def test_model_apply_matches_oracle(family, dtype, hf_models):
    _, cfg, params = hf_models[family]
    model = CLASSES[family](cfg, dtype=dtype)
    g = torch.Generator().manual_seed(5)
    ids = torch.randint(0, cfg.vocab_size, (3, 9), generator=g, dtype=torch.int32)
    want = O.forward(family, cfg, params, ids, dtype).logits
    out = model.apply(params, ids)
    assert tuple(out.logits.shape) == (3, 9, cfg.vocab_size) and out.logits.dtype == dtype
    _close(out.logits, want, dtype)
    last = model.apply(params, ids, keep_last_n_logits=2).logits
    assert tuple(last.shape) == (3, 2, cfg.vocab_size)
    _close(last, want[:, -2:], dtype)
    if dtype == torch.float32:
        mask = torch.ones(3, 9, dtype=torch.bool)
        mask[1, 6:] = False
        got = model.apply(params, ids, attention_mask=mask).logits
        ref = O.forward(family, cfg, params, ids, dtype, attention_mask=mask).logits
        _close(got[0], ref[0], dtype)
        _close(got[1, :6], ref[1, :6], dtype)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16], ids=["f32", "bf16"])
@pytest.mark.parametrize("family", ["llama", "neox", "gemma3"])
def test_stack_model_apply_matches_oracle(family, dtype, hf_models):
    """``*Model.apply``: the final-norm hidden states of every position against the oracle's."""
    from jaxml_b200.models import GemmaModel, GPTNeoXModel, LlamaModel

    _, cfg, params = hf_models[family]
    cls = {"llama": LlamaModel, "neox": GPTNeoXModel, "gemma3": GemmaModel}[family]
    body = "gpt_neox" if family == "neox" else "model"
    model = cls(cfg, dtype=dtype)
    g = torch.Generator().manual_seed(6)
    ids = torch.randint(0, cfg.vocab_size, (2, 11), generator=g, dtype=torch.int32)
    want = O.forward(family, cfg, params, ids, dtype).last_hidden_state
    out = model.apply({"params": params["params"][body]}, ids).last_hidden_state
    assert tuple(out.shape) == (2, 11, cfg.hidden_size) and out.dtype == dtype
    _close(out, want, dtype)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16], ids=["f32", "bf16"])
@pytest.mark.parametrize("family", ["llama", "neox", "gemma3"])
def test_apply_with_kv_caches_matches_oracle(family, dtype, hf_models):
    """A right-padded prompt into empty ``KVCache`` objects, then one token per row into the populated
    caches, through ``*ModelWithHead.apply`` (the decoder blocks), against the oracle's cached forward:
    logits, cache contents, masks and positions."""
    from jaxml_b200.cache import KVCache

    _, cfg, params = hf_models[family]
    model = CLASSES[family](cfg, dtype=dtype)
    L, T = cfg.num_layers, 16
    g = torch.Generator().manual_seed(7)
    ids = torch.randint(0, cfg.vocab_size, (2, 6), generator=g, dtype=torch.int32)
    mask = torch.ones(2, 6, dtype=torch.bool)
    mask[1, 4:] = False
    out = model.apply(params, ids, attention_mask=mask, kv_caches=tuple(KVCache.init(T, dtype=dtype) for _ in range(L)),
                      use_cache=True)
    ref = O.forward(family, cfg, params, ids, dtype, attention_mask=mask,
                    kv_caches=[O.OracleKVCache(T, dtype) for _ in range(L)])
    _close(out.logits[0], ref.logits[0], dtype)
    _close(out.logits[1, :4], ref.logits[1, :4], dtype)
    caches, ocaches = out.kv_caches, ref.kv_caches
    for step in range(4):
        for c, oc in zip(caches, ocaches):
            assert torch.equal(c.mask.cpu(), oc.mask)
            assert torch.equal(c.pos_id.cpu().long(), oc.pos_id.long())
            _close(c.k, oc.k, dtype)
            _close(c.v, oc.v, dtype)
        if step == 3:
            break
        nxt = torch.randint(0, cfg.vocab_size, (2, 1), generator=g, dtype=torch.int32)
        out = model.apply(params, nxt, kv_caches=caches, use_cache=True)
        ref = O.forward(family, cfg, params, nxt, dtype, kv_caches=list(ocaches))
        assert tuple(out.logits.shape) == (2, 1, cfg.vocab_size)
        _close(out.logits, ref.logits, dtype)
        caches, ocaches = out.kv_caches, ref.kv_caches


@pytest.mark.parametrize("family", ["llama", "neox", "gemma3"])
def test_apply_hidden_states_and_position_ids(family, hf_models):
    """``output_hidden_states`` (every layer's input, then the final-norm output), ``use_cache`` without
    caches, and explicit (broadcast) position ids, against the oracle."""
    from jaxml_b200.models import GemmaModel, GPTNeoXModel, LlamaModel

    _, cfg, params = hf_models[family]
    dtype = torch.float32
    model = CLASSES[family](cfg, dtype=dtype)
    g = torch.Generator().manual_seed(8)
    ids = torch.randint(0, cfg.vocab_size, (2, 5), generator=g, dtype=torch.int32)
    ref = O.forward(family, cfg, params, ids, dtype)
    out = model.apply(params, ids, output_hidden_states=True, use_cache=True)
    assert out.kv_caches == (None,) * cfg.num_layers
    assert len(out.hidden_states) == cfg.num_layers + 1
    for got, want in zip(out.hidden_states, ref.hidden_states):
        _close(got, want, dtype)
    _close(out.logits, ref.logits, dtype)
    stack = {"llama": LlamaModel, "neox": GPTNeoXModel, "gemma3": GemmaModel}[family](cfg, dtype=dtype)
    body = params["params"]["gpt_neox" if family == "neox" else "model"]
    sout = stack.apply({"params": body}, ids, output_hidden_states=True)
    _close(sout.last_hidden_state, ref.last_hidden_state, dtype)
    assert len(sout.hidden_states) == cfg.num_layers + 1 and sout.kv_caches is None
    pos = torch.arange(5, dtype=torch.int32)[None] + 3
    ref = O.forward(family, cfg, params, ids, dtype, position_ids=pos.expand(2, 5))
    out = model.apply(params, ids, position_ids=pos)
    _close(out.logits, ref.logits, dtype)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16], ids=["f32", "bf16"])
@pytest.mark.parametrize("family", ["llama", "neox", "gemma3"])
def test_mlp_blocks_match_oracle(family, dtype, hf_models):
    """``LlamaMLP`` / ``GPTNeoXMLP`` / ``GemmaMLP`` (projections + ``jx_mlp_act``) against the oracle's MLP."""
    from jaxml_b200.models import GemmaMLP, GPTNeoXMLP, LlamaMLP

    _, cfg, params = hf_models[family]
    lp = params["params"]["gpt_neox" if family == "neox" else "model"]["layers_0"]
    cls = {"llama": LlamaMLP, "neox": GPTNeoXMLP, "gemma3": GemmaMLP}[family]
    g = torch.Generator().manual_seed(9)
    x = torch.randn(2, 3, cfg.hidden_size, generator=g).to(dtype)
    mp = {k: {kk: torch.as_tensor(vv).cuda() for kk, vv in v.items()} for k, v in lp["mlp"].items()}
    got = cls(cfg, dtype=dtype).apply({"params": mp}, x.cuda())
    want = O._mlp(family, lp, x, dtype)
    assert got.dtype == dtype and tuple(got.shape) == (2, 3, cfg.hidden_size)
    _close(got, want, dtype)


def test_engine_step_interface_matches_generate(hf_models):
    """``Engine.init_cache`` + ``Engine.wrapped_apply_fn`` (the reference's step-by-step decoding,
    engine.py:110-121 and 355-377): last-position logits against the oracle, and greedy steps that give
    the tokens ``Engine.generate`` (the fused runtime) gives."""
    from jaxml_b200 import Engine, InferenceConfig

    _, cfg, params = hf_models["llama"]
    model = CLASSES["llama"](cfg)
    eng = Engine(model, InferenceConfig(), params)
    g = torch.Generator().manual_seed(10)
    ids = torch.randint(0, cfg.vocab_size, (2, 5), generator=g, dtype=torch.int32)
    logits, caches = eng.wrapped_apply_fn(params, ids, kv_caches=eng.init_cache(16))
    assert tuple(logits.shape) == (2, 1, cfg.vocab_size) and len(caches) == cfg.num_layers
    _close(logits[:, 0], O.forward("llama", cfg, params, ids, torch.float32).logits[:, -1], torch.float32)
    toks = []
    for _ in range(4):
        nxt = logits[:, -1].argmax(-1, keepdim=True).to(torch.int32)
        toks.append(nxt.cpu())
        logits, caches = eng.wrapped_apply_fn(params, nxt, kv_caches=caches)
    want = eng.generate(ids, max_new_tokens=4, temperature=0.0, include_prompt=False)
    assert torch.equal(torch.cat(toks, 1), torch.as_tensor(want).cpu().to(torch.int32))
    eng.close()


@pytest.mark.parametrize("family", ["llama", "gemma3"])
def test_apply_output_attentions(family, hf_models):
    """``output_attentions``: one [B, H, S, S] probability array per layer (causal, rows summing to one, the
    sliding window on Gemma's local layers), with logits unchanged against the oracle."""
    _, cfg, params = hf_models[family]
    model = CLASSES[family](cfg)
    g = torch.Generator().manual_seed(11)
    ids = torch.randint(0, cfg.vocab_size, (2, 7), generator=g, dtype=torch.int32)
    out = model.apply(params, ids, output_attentions=True)
    _close(out.logits, O.forward(family, cfg, params, ids, torch.float32).logits, torch.float32)
    assert len(out.attention_weights) == cfg.num_layers
    upper = torch.triu(torch.ones(7, 7, dtype=torch.bool), 1)
    for li, w in enumerate(out.attention_weights):
        w = w.float().cpu()
        assert tuple(w.shape) == (2, cfg.num_heads, 7, 7)
        assert torch.allclose(w.sum(-1), torch.ones(2, cfg.num_heads, 7), atol=1e-5)
        assert bool((w[..., upper] == 0).all())
        if family == "gemma3" and (li + 1) % cfg.sliding_window_pattern:
            lower = torch.tril(torch.ones(7, 7, dtype=torch.bool), -cfg.sliding_window)
            assert bool((w[..., lower] == 0).all())
