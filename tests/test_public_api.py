"""The reference's import paths and names (``tests/test_public_api.py`` of the reference) resolve to the
same objects here."""


def test_root_and_inference_engine_exports():
    import jaxml_b200 as root
    from jaxml_b200 import inference_engine as ie
    from jaxml_b200.config import ModelConfig
    from jaxml_b200.engine import Engine, InferenceConfig
    from jaxml_b200.sampling import SamplingMethod
    from jaxml_b200.text_generation import GenerationConfig, TextGenerationPipeline

    assert ie.Engine is Engine and ie.InferenceConfig is InferenceConfig and ie.SamplingMethod is SamplingMethod
    assert root.Engine is Engine and root.InferenceConfig is InferenceConfig and root.ModelConfig is ModelConfig
    assert root.SamplingMethod is SamplingMethod and root.GenerationConfig is GenerationConfig
    assert root.TextGenerationPipeline is TextGenerationPipeline


def test_nn_and_outputs_exports():
    from jaxml_b200 import nn, outputs

    for name in ("Attention", "AttentionWithRoPE", "Block", "DenseGeneral", "Embed", "LayerNorm", "Module",
                 "RMSNorm", "RotaryEmbedding"):
        assert hasattr(nn, name), name
    for name in ("AttentionOutput", "BaseModelOutputWithCache", "CausalLMOutputWithCache", "DecoderOutput",
                 "GenerationOutput"):
        assert hasattr(outputs, name), name
    assert outputs.AttentionOutput is nn.AttentionOutput


def test_model_classes():
    from jaxml_b200 import GemmaModelWithHead, GPTNeoXModelWithHead, LlamaModelWithHead, models

    assert models.LlamaModelWithHead is LlamaModelWithHead and models.GemmaModelWithHead is GemmaModelWithHead
    assert models.GPTNeoXModelWithHead is GPTNeoXModelWithHead
    assert models.CausalLMOutputWithCache.__name__ == "CausalLMOutputWithCache"
