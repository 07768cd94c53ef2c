"""macai_b200: the chunked gated delta rule (Qwen3.5 / Qwen3-Next linear attention) as hand-written sm_100a (B200)
CUDA kernels behind a C ABI, with the reference package's Python surface (AbstractEyes/Mac-ai-engineering, `macai`):

    from macai_b200.gated_delta import chunk_gated_delta_rule     # drop-in for transformers' torch_chunk_gated_delta_rule
    import macai_b200.patch; macai_b200.patch.install()            # route transformers' Qwen3.5-family models to it
"""
__version__ = "0.1.0"
