"""Drop-in replacements for the reference's relative-position attention kernels.

Same module paths and call signatures as vllm-factory's `kernels.flash_attention_rpb`
and `kernels.flash_deberta_attention`; the work runs in the sm_100a kernels of
libvf_b200.so through torch.ops.vf_b200.*.
"""
