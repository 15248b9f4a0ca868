"""``install_into_reference`` inside the reference's own model code (CPU).

The reference imports its layer operator into ``llada/model/modeling_llada.py``
(line 55) and calls it from ``LLaDABlock.attention`` (line 760).  This test
imports the reference's model module from a local checkout (skipped where
there is none: the checkout never travels to the GPU box), rebinds the
operator with ``install_into_reference`` and runs a forward of a tiny
reference ``LLaDAModelLM`` with Flash-Cache arguments built by the
reference's own ``make_blocks``.  On the CPU this package's operator refuses
the CPU tensors ("no CPU path"); reaching that refusal proves the reference's
forward routes every layer through this package with the reference's
argument lists.  The GPU run of the operator on those argument lists is
``tests/test_layer_gpu.py::test_drop_in_matches_the_reference_layer_run``.
"""
import os
import sys

import pytest
import torch

REF = os.environ.get("FDLLM_REFERENCE_DIR", "/root/reference/llada")


@pytest.mark.skipif(not os.path.isdir(REF), reason="no reference checkout")
def test_install_routes_the_reference_forward_through_this_package():
    import cases
    sys.path.insert(0, REF)
    try:
        import model.modeling_llada as ml
        from model.configuration_llada import LLaDAConfig
    finally:
        sys.path.remove(REF)
    from flash_dllm_b200.flash_cache import flash_fused_elastic_cache, install_into_reference
    original = ml.flash_fused_elastic_cache
    cfg, w = cases.gen_weights()
    rc = LLaDAConfig(d_model=cfg.d_model, n_heads=cfg.n_heads, n_layers=cfg.n_layers,
                     mlp_hidden_size=cfg.mlp_hidden_size, vocab_size=cfg.vocab_size, embedding_size=cfg.vocab_size,
                     weight_tying=False, block_type="llama", layer_norm_type="rms", activation_type="silu",
                     rope=True, rope_theta=cfg.rope_theta, rms_norm_eps=cfg.rms_norm_eps, include_bias=False,
                     residual_dropout=0.0, embedding_dropout=0.0, attention_dropout=0.0, flash_attention=False,
                     init_device="cpu", max_sequence_length=4096)
    m = ml.LLaDAModelLM(rc, init_params=False)
    m.load_state_dict(w, strict=True)
    m = m.to(torch.bfloat16)
    calls = []

    def spy(*a, **k):
        calls.append(a[0])
        return flash_fused_elastic_cache(*a, **k)

    try:
        install_into_reference(ml)
        assert ml.flash_fused_elastic_cache is flash_fused_elastic_cache
        ml.flash_fused_elastic_cache = spy  # same routing, counting the calls
        c = cases.cache_case()
        L = cases.LMAX
        for blk in m.model.transformer.blocks:
            blk.k_cache, blk.v_cache = c["k_cache"].bfloat16(), c["v_cache"].bfloat16()
        qb = torch.cat([c["masked_blocks"], c["tracked_blocks"]])
        positions = [c["pos"], torch.tensor([], dtype=torch.int64), [c["sin"], c["cos"]], [], torch.zeros(2 * L), []]
        lengths = [[-1, -1], None, c["masked_blocks"], c["tracked_blocks"], qb, [0, 1], 2, L, cases.BLOCK_M, 128,
                   None, False]
        ids = torch.randint(0, cfg.vocab_size, (1, c["pos"].numel()))
        with pytest.raises(ValueError, match="CUDA tensor"):
            with torch.no_grad():
                m(ids, use_cache=True, lengths=lengths, positions=positions)
        assert len(calls) == 1 and calls[0] is m.model.transformer.blocks[0]
    finally:
        ml.flash_fused_elastic_cache = original
