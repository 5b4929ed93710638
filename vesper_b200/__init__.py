"""vesper_b200: B200-native (sm_100a) kernels for the column hot path of mstampfli/vesper-preview.

The package mirrors the reference's entry points for that path (``vesper.kernels.delta_scan``,
``vesper.kernels.keys``, ``vesper.kernels.norm``, ``vesper.kernels.window_attn``) and runs them as
hand-written CUDA through the C ABI of ``libvesper_b200.so`` (``include/vesper_b200.h``).
"""

from vesper_b200.contracts import ContractError

__all__ = ["ContractError"]
