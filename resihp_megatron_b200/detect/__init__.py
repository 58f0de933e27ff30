"""L7 fail-slow detection: gated RLS predictor, residual BOCD, ski-rental policy, the
coordinator-side DetectorService, chunk timers, validation probes, synthetic traces, and the
native NCCL profiler plugin with its ring reader."""
