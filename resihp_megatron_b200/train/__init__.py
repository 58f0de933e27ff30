"""L6 training: the resilient loop and its runtime bindings (replica DP, heterogeneous hybrid
parallel on the CPU reference model, and the GPU engine)."""
