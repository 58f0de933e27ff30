"""L3 communication: generation-scoped communicators (shrink / split / fresh, abortable waits),
plan-derived group specs, heterogeneous pipeline-boundary P2P, and the per-generation symmetric
peer-memory heap used by the fused kernels."""
