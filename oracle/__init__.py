"""CPU oracle for the quantized SmolVLA ``sample_actions`` path.

TEST INFRASTRUCTURE ONLY.  Nothing in the product package imports this
package.  Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline
leg of ``bench.py`` use it, and only as the checker or as the timed
CPU baseline, never as the thing that is measured or shipped.

Contents
--------
quant    restatement of the SmoothQuant fake-dequant arithmetic of the
         reference (deploy/linear_only_quant.py:40-172,
         deploy/build_smoothquant_scales.py:55-106,
         deploy/calibrate_smolvla_activation_channel_scales.py:53-134).
         Pinned against the reference's own code by tests/golden/ fixtures
         produced by tests/golden/make_golden.py, which imports the reference
         modules unchanged.
model    restatement of the SmolVLA core (prefix embed, masks, SigLIP +
         connector, SmolVLM2 text layers, action expert, flow-matching loop).
         The model code lives in lerobot 0.5.1, which is not shipped with the
         reference, so for the lerobot-resident pieces parity is UNPINNED;
         the arithmetic follows the reference's restatements in
         deploy/diagnose_3_4_numeric_baseline.py:42-206,
         deploy/export_6f_layer0_attention_tensors.py:100-119 and
         deploy/validate_fused_rope_layout_math.py:28-42.
metrics  compare_tensors semantics of deploy/diagnose_3_4_numeric_baseline.py:806-834.
"""
