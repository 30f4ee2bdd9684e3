"""Row shims of the DiT, the same modules, names and signatures as
``h3_inference/kernels`` (``__init__.py:1-13``), calling this library's
sm_100a kernels where the reference's env flags arm them.

``_dispatch`` also stands in for the reference's plug-in package: its
``try_call(name, *args)`` answers the names the reference's own shims ask
for, so either the model imports these modules or the reference's modules
reach the kernels through ``try_call`` (see ``_dispatch``)."""
from h3_engine_b200.kernels import (
    elementwise_norm_rope,
    ffn_qkvo_gemms,
    other,
    packed_self_attn,
)

__all__ = [
    "elementwise_norm_rope",
    "ffn_qkvo_gemms",
    "other",
    "packed_self_attn",
]
