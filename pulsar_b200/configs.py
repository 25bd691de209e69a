"""The five BASELINE configurations as LayerSpecs (seeded synthetic data).

C1  hidden 2048, 128 experts, softmax top-8, F 768, Q4_K, Zipf(1.1) logit bias
C2  hidden 2048, 256 experts, sigmoid top-8 + 1 shared, F 512, all Q4_K,
    Zipf(1.1) selection bias, 40 layers
C3  hidden 2880, 32 experts, softmax top-4, F 2880, MXFP4, biases N(0, 0.01),
    swiglu_oai (gpt-oss)
C4  hidden 4096, 128 experts, softmax top-8, F 1536, Q2_K, Zipf(1.2), 94 layers
C5  hidden 7168, 256 experts, sigmoid top-8 group-limited (8 groups, top 4)
    + 1 shared Q8_0, F 2048, IQ2_XXS (uniform importance), 61 layers
"""
from ._lib import QUANT_IQ2_XXS, QUANT_MXFP4, QUANT_Q2_K, QUANT_Q4_K, QUANT_Q8_0
from .layer import LayerSpec

CONFIGS = {
    "C1": dict(spec=LayerSpec(n_embd=2048, n_ff=768, n_expert=128, n_used=8, quant=QUANT_Q4_K, router_mode=1,
                              zipf_s=1.1, zipf_kind="logit"), layers=1, batches=(1,)),
    "C2": dict(spec=LayerSpec(n_embd=2048, n_ff=512, n_expert=256, n_used=8, quant=QUANT_Q4_K, router_mode=0,
                              zipf_s=1.1, zipf_kind="select", shared_quant=QUANT_Q4_K, shared_n_ff=512),
               layers=40, batches=(1, 8, 64)),
    "C3": dict(spec=LayerSpec(n_embd=2880, n_ff=2880, n_expert=32, n_used=4, quant=QUANT_MXFP4, router_mode=1,
                              act_op=2, biases=True), layers=1, batches=(1, 2048)),
    "C4": dict(spec=LayerSpec(n_embd=4096, n_ff=1536, n_expert=128, n_used=8, quant=QUANT_Q2_K, router_mode=1,
                              zipf_s=1.2, zipf_kind="logit", router_q8_0=True), layers=94, batches=(1, 32, 256)),
    "C5": dict(spec=LayerSpec(n_embd=7168, n_ff=2048, n_expert=256, n_used=8, quant=QUANT_IQ2_XXS, router_mode=0,
                              n_group=8, topk_group=4, zipf_s=1.1, zipf_kind="select", shared_quant=QUANT_Q8_0,
                              shared_n_ff=2048), layers=61, batches=(4096, 64)),
}


def scaled(spec: LayerSpec, n_expert=None, n_embd=None, n_ff=None, shared_n_ff=None) -> LayerSpec:
    """A smaller layer of the same structure (parity tests)."""
    from dataclasses import replace
    kw = {}
    if n_expert is not None:
        kw["n_expert"] = n_expert
    if n_embd is not None:
        kw["n_embd"] = n_embd
    if n_ff is not None:
        kw["n_ff"] = n_ff
    if shared_n_ff is not None:
        kw["shared_n_ff"] = shared_n_ff
    return replace(spec, **kw)
