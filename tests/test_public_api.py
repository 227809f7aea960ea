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

    assert nn.__all__ == ["Attention", "AttentionWithRoPE", "Block", "DenseGeneral", "Embed", "LayerNorm", "Module",
                          "RMSNorm", "RotaryEmbedding"]
    for name in nn.__all__:
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


def test_models_module_exports_architecture_entry_points():
    import jaxml_b200.models as models

    assert models.__all__ == ["GPTNeoXDecoder", "GPTNeoXMLP", "GPTNeoXModel", "GPTNeoXModelWithHead", "GemmaDecoder",
                              "GemmaMLP", "GemmaModel", "GemmaModelWithHead", "GemmaRMSNorm", "LlamaDecoder",
                              "LlamaMLP", "LlamaModel", "LlamaModelWithHead"]
    for name in models.__all__:
        assert isinstance(getattr(models, name), type), name
    from jaxml_b200.decoders import LlamaDecoder
    from jaxml_b200.nn import GemmaRMSNorm

    assert models.LlamaDecoder is LlamaDecoder and models.GemmaRMSNorm is GemmaRMSNorm


def test_importing_the_package_leaves_root_logging_alone():
    import importlib
    import logging
    import sys

    root = logging.getLogger()
    handlers, level = list(root.handlers), root.level
    saved = {k: v for k, v in sys.modules.items() if k == "jaxml_b200" or k.startswith("jaxml_b200.")}
    for k in saved:
        sys.modules.pop(k)
    root.handlers.clear()
    root.setLevel(logging.WARNING)
    try:
        importlib.import_module("jaxml_b200")
        assert root.handlers == [] and root.level == logging.WARNING
    finally:
        for k in [k for k in sys.modules if k == "jaxml_b200" or k.startswith("jaxml_b200.")]:
            sys.modules.pop(k)
        sys.modules.update(saved)
        root.handlers[:] = handlers
        root.setLevel(level)


def test_inference_engine_submodules():
    from jaxml_b200.engine import Engine as E
    from jaxml_b200.inference_engine.engine import Engine, InferenceConfig
    from jaxml_b200.inference_engine.sampling import SamplingMethod, top_k_filtering
    from jaxml_b200.sampling import SamplingMethod as S

    assert Engine is E and SamplingMethod is S and callable(top_k_filtering) and InferenceConfig is not None
