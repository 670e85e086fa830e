"""Decoder model pieces: attention, SwiGLU MLP, blocks, paged KV cache."""
