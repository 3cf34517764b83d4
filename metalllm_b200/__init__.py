"""B200 (sm_100a) implementation of metalLLM's causal attention hot path.

Modules (imported on demand; this package imports nothing at load time):
    attention  the reference's four attention operators, the GEMMs around
               them, the fused variants and HostPipeline, on torch CUDA
               tensors through libmetalattn's C ABI
    train      TrainingModel, the config-5 training step (model.h's Model)
    shards     (batch, head) shard plans for several GPUs
    inputs     the deterministic synthetic input generator
    build      compiles libmetalattn.so (and the CPU oracle) in-tree
"""
