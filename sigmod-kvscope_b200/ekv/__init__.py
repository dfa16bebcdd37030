"""ekv on B200: the attention-share audit and block-table view path of KVScope, on sm_100a kernels.

The subpackages mirror the reference's module paths (``runtime.audit_kernel``,
``runtime.block_view``, ``observe.tile_shares``, ``observe.allocation``, ``observe.ranks``) with the
same names, signatures and exceptions, so a caller switches by importing ``ekv.runtime`` and
``ekv.observe`` in their place. Every device computation runs in ``libekv_b200.so`` (``ekv._lib``).
"""

__version__ = "0.1.0"
