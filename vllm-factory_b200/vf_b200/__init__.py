"""vf_b200 — B200-native (sm_100a) relative-position encoder attention for vllm-factory.

`import vf_b200.ops` loads the kernel library (libvf_b200.so) and the torch op layer
(libvf_b200_torch.so) and registers torch.ops.vf_b200.rpb_attention and
torch.ops.vf_b200.deberta_attention.  The drop-in modules with the reference's call
signatures live in the sibling `kernels` package (kernels.flash_attention_rpb,
kernels.flash_deberta_attention): put the `vllm-factory_b200` directory on sys.path ahead
of the reference checkout and the reference's models resolve to them.
"""
from ._lib import device_error, load  # noqa: F401

__all__ = ["load", "device_error"]
