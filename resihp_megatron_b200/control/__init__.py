"""L1 control plane: coordinator (generations, transactions, fencing, HA), node agents,
in-worker client, KV store, membership, health probes and the ``resihp-run`` launcher."""

from .coordinator import ClusterView, Coordinator, PlannerFn, keep_all_planner  # noqa: F401
from .kvstore import InMemoryKV, KVStore  # noqa: F401
from .membership import Membership, WorkerRecord, WorkerState  # noqa: F401
