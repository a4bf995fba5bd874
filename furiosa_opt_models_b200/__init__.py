"""Model implementations, kernels and parallel runtime behind ``furiosa_opt_engine``.

- ``ops``: Python handles on the sm_100a kernels (raw launchers of the native extension) and the
  PyTorch reference math each kernel is tested against.
- ``models``: model configs, the checkpoint-driven decoders (Qwen3, Llama, Mistral, Qwen3-MoE) and
  their CPU reference path.
- ``parallel``: tensor and expert parallelism: peer memory, fused collectives, rank plumbing.
- ``utils``: the native build, tracing and environment handling.
"""
