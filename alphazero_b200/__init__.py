"""B200-native evaluation backend for the residual policy/value network of
tianjianh/AlphaZero ("MiniGo C++"): the batched forward pass behind
``InferenceEngine::predict_batch`` as hand-written sm_100a kernels behind a
C ABI (include/minigo_cuda.h)."""


def __getattr__(name):
    if name == "CudaEngine":
        from .engine import CudaEngine
        return CudaEngine
    raise AttributeError(name)
