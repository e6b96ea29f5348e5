"""knurlogic_b200: the VQ-quantised MoE expert layer of Knurlogic, on B200.

Drop-in modules with the reference's interface (`VQSwitchLinear`,
`SwitchLinear`, `SwitchGLU`, `SparseMoeBlock`) over libvqmoe.so, hand-written
sm_100a CUDA behind a C ABI (include/vqmoe.h). Tensor parallelism follows
the reference's split rules (`tensor_split`).
"""
from .switch_layers import (GeGLU, QuantizedSwitchLinear, SwiGLU, SwitchGLU, SwitchLinear,  # noqa: F401
                            VQSwitchLinear)
from .moe import CapturedBlock, SharedExpert, SparseMoeBlock  # noqa: F401
from . import gemma4  # noqa: F401

__all__ = ["SwitchGLU", "SwitchLinear", "VQSwitchLinear", "QuantizedSwitchLinear", "SwiGLU", "GeGLU",
           "SharedExpert", "CapturedBlock", "SparseMoeBlock"]
