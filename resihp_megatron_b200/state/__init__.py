"""L5 state: transactions and roll-forward, slice transfer planning and execution, resharding
checkpoints (T2), host snapshots (T1), warm handoff, placement-independent RNG and data."""
