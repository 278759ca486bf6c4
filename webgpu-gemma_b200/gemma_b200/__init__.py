"""gemma_b200: B200-native Gemma 3 Q8_0 token loop (host side).

The compute path is libgemma_b200.so (hand-written CUDA for sm_100a behind a C-ABI,
declared in include/gemma_b200.h). This package is the host-side mirror of the
reference's TypeScript surface (createGemmaEngine / addUserMessage / generate /
resetConversation / dispose) plus its GGUF parser, tokenizer and chat template.
"""
from .config import GemmaConfig, default_config, get_rope_theta, is_swa_layer  # noqa: F401
