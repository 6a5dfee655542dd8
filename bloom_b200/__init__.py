"""bloom_b200: a B200-native (sm_100a) inference engine with the capabilities of Bloom.

Layers (bottom-up):
  _C / ops        hand-written sm_100a kernels (tcgen05 GEMM, paged attention, norms, RoPE, sampling)
  _runtime        C++ host runtime (KV block manager, in-flight batching scheduler, CPU GGUF kernels)
  models          decoder LMs (Llama / Qwen2 / Qwen3 / Mistral), Qwen3-MoE, BERT encoders
  parallel        tensor / expert / data parallelism over NVLink (NCCL plumbing + fused kernels)
  engine          model runner (CUDA graphs), LLMEngine (public generate API), speculative decoding
  formats         GGUF, safetensors, bloom.json manifests, memory estimator
  server / cli    OpenAI- and Ollama-compatible HTTP server, bloom_infer / bloom_bench CLIs
"""

__version__ = "0.1.0"
