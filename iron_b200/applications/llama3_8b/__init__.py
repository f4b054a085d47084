"""Llama-3-8B-shaped decoder block, tensor-parallel over NCCL (one node)."""
