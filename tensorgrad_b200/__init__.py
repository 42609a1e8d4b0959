"""tensorgrad_b200 — tensorgrad's training API on a B200-native CUDA backend.

The graph layer (IR, tracer, ops, autograd, DCE, optimizers, LR schedules,
modules) mirrors the reference's TypeScript library; everything below the
traced graph runs in libtgcuda.so (hand-written sm_100a kernels, C ABI in
include/tensorgrad_b200.h).
"""
from .ir import Graph, Tensor
from .trace import trace_fn as traceFn, trace_into as traceInto, param_input as paramInput, \
    tensor_input as tensorInput, state_input as stateInput
from .ops import *  # noqa: F401,F403
from .ops import sum, min, max, abs  # noqa: F401,A004
from .module import Module, init, mulberry32
from .nn import Linear, LayerNorm, RMSNorm, Embedding, Conv2d, crossEntropy, nllLoss
from .lr import lr, resolveLR
from .grad import appendGrad, appendGradClip, appendGradNormalize
from .dce import eliminateDeadCode
from .optim import appendAdam, appendSGD, adamStepScalars
from .shape import ShapeError
from .compile import compile, compileForward, trace, CompiledTraining, CompiledForward  # noqa: A004
from .safetensors import loadSafetensors, saveSafetensors
