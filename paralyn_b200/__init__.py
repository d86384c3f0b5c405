"""paralyn_b200: a B200-native (sm_100a) implementation of Paralyn's FP32
operator path behind the reference's native C ABI.

The Python surface mirrors the reference binding (package `paralyn`): Context,
Buffer, View, Module, Kernel, Queue, Event, asarray/add/affine, tensor/matmul/
layer_norm/residual_add/bias_add, with the same status codes and errors. The
compute runs in libparalyn_native.so (C++17 runtime + hand-written CUDA kernels
for sm_100a); there is no CPU fallback.
"""
__version__ = "0.1.0"

from .native import (ABI_VERSION, ARTIFACT_MSL_SOURCE, ARTIFACT_SPIRV_MSL, ARTIFACT_VERIFIED_IR,
                     Access, BackendStatus, Buffer, ClockDomain, Context, Device,
                     DeviceCapabilities, Error, Event, EventInfo, EventTiming, Kernel, Module,
                     Parameter, Queue, Scalar, Status, Type, View, backend_status,
                     device_capabilities, devices, f32, i32, library, u32)
from .array import Array, add, affine, affine_scalar, asarray, float32
from .tensor import (Activation, Reduce, Tensor, TensorDescriptor, TensorOperatorCapabilities,
                     add_into, batched_matmul, batched_matmul_into, bias_activation_into, bias_add,
                     bias_gelu, gelu, layer_norm, layer_norm_into, load_tensor_operators, matmul,
                     matmul_into, reduce_rows_into, relu, residual_add, row_max, row_sum, softmax,
                     softmax_rows_into, tensor, tensor_operators_artifact,
                     tensor_operators_capabilities)
from .b200 import (MatmulMode, device_kernel_count, fill_synthetic_into, inspect_module, matmul_mode,
                   set_matmul_mode)
