"""Parallel layouts: expert parallelism over NVLink peer memory, ZeRO-1 data
parallelism, tensor/sequence and pipeline parallelism."""
