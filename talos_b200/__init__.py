"""talos_b200 -- the B200 (sm_100a) decode path for Talos GGUF/Llama models.

Public API (mirrors Tsuskov/talos ``src/model`` for the CUDA backend):
    Model.load(path) / Model.load_bytes(data)
    Model.forward_gpu / forward_hidden_gpu / step / step_hidden / reset / cap_context
    Model.generate_greedy / prefill
    Model.set_batch / forward_batch / prefill_slot / generate_batch_greedy  (batches)
    argmax, dequant, matvec, Weight   (single-kernel entry points)
The compute runs in libtalos_cuda.so through the C ABI of include/talos_cuda.h.
"""
from .gguf import F32, Q4_0, Q6_K, Q8_0, GgufError, GgufFile, GgufWriter, TensorInfo
from .model import Config, Context, Model, Weight, argmax, dequant, matvec, nccl_unique_id, weight_shapes

__all__ = ["F32", "Q4_0", "Q6_K", "Q8_0", "GgufError", "GgufFile", "GgufWriter", "TensorInfo", "Config",
           "Context", "Model", "Weight", "argmax", "dequant", "matvec", "nccl_unique_id", "weight_shapes"]
