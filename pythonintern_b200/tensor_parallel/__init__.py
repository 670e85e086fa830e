"""Tensor-parallel primitives: linears, RMSNorm, NVLink all-reduce, weight sharding."""
