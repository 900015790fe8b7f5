"""smelt_b200: B200-native (sm_100a) GPT-2 forward over group-quantized weights.

The hot path of LukasParke/smelt's model-lab (the GPT-2 forward its own CUDA
kernels compute) rebuilt as precompiled CUDA kernels behind the C-ABI of
include/gpt2q.h. Python modules:
  atoms  - SMT numeric atoms (f16 codec, Q8 / int4 group quantisers)
  pack   - converter policy and tensor records (the weight-layout boundary)
  synth  - seeded synthetic weights and token ids
  gpu    - `Gpu`, the mirror of model-lab's Gpu::new / step / clear_kv
"""
from .pack import CONFIGS, GPT2_MEDIUM, GPT2_SMALL, GPT2_XL, Meta, Pack, from_hf  # noqa: F401

__all__ = ["CONFIGS", "GPT2_SMALL", "GPT2_MEDIUM", "GPT2_XL", "Meta", "Pack", "from_hf"]
