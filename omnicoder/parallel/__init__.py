"""Parallel layouts: expert parallelism over NVLink peer memory, ZeRO-1 data
parallelism, tensor/sequence, context (all-to-all over heads) and pipeline parallelism."""
