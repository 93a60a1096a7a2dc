"""chonklm_b200: a B200-native (sm_100a) decode engine for small GGUF decoder
models, behind the module API of ChonkLM's llama-webgpu runtime."""
