"""Baselines the fused collective is measured against (NCCL, vLLM, FlashInfer, the reference prototype)."""
