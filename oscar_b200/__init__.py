"""oscar_b200: a Blackwell-native (sm_100a) serving framework for Qwen3.5-shaped hybrid
models with an INT2 KV cache and MTP speculative decoding.

``LLM`` / ``SamplingParams`` are the offline generation API; ``python -m oscar_b200.serve``
the HTTP server.
"""


def __getattr__(name):
    # lazy: importing the package must not import torch-heavy modules (the build step
    # imports it before the extension exists)
    if name == "LLM":
        from .llm import LLM
        return LLM
    if name == "SamplingParams":
        from .ops.sampling import SamplingParams
        return SamplingParams
    raise AttributeError(name)
