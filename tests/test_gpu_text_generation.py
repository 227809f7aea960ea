"""TextGenerationPipeline.from_hf end to end on the GPU: a tiny HF Llama saved to disk, loaded through
the reference's parameter tree, packed for this GPU, greedy tokens identical to the oracle's (float32)."""
import numpy as np
import pytest
import torch

from tests.test_text_generation import _Tok

pytestmark = pytest.mark.gpu


def test_from_hf_greedy_tokens_match_oracle(tmp_path):
    from transformers import LlamaConfig, LlamaForCausalLM

    from jaxml_b200 import TextGenerationPipeline
    from oracle import jaxml_oracle as O

    torch.manual_seed(0)
    hf_cfg = LlamaConfig(hidden_size=256, intermediate_size=512, num_hidden_layers=2, num_attention_heads=4,
                         num_key_value_heads=2, vocab_size=512, max_position_embeddings=1024, rms_norm_eps=1e-5)
    LlamaForCausalLM(hf_cfg).save_pretrained(tmp_path)
    pipe = TextGenerationPipeline.from_hf(tmp_path, tokenizer=_Tok())
    prompts = ["hello world", "b200"]
    toks = pipe.generate_tokens(prompts, max_new_tokens=6, temperature=0.0, include_prompt=False)
    enc = _Tok()(prompts)
    ids, mask = enc["input_ids"], enc["attention_mask"].astype(bool)
    model = pipe.engine.model
    want = O.generate("llama", model.config, pipe.engine.params, torch.as_tensor(ids), torch.float32,
                      max_new_tokens=6, temperature=0.0, attention_mask=torch.as_tensor(mask), include_prompt=False)
    assert np.array_equal(toks, np.asarray(want)), (toks, want)
    text = pipe.generate_text("hello", max_new_tokens=3, temperature=0.0)
    assert isinstance(text, str) and len(text) == len("hello") + 3
    pipe.engine.close()
