"""L4 runtime: float64 reference models (semantic oracles), pipeline IR interpreter,
heterogeneous runtime and shard-aligned grad sync, replica-DP runtime, MoE expert parallelism,
Adam, zero-bubble weight-gradient stores and per-generation hooks."""
