"""Named planner instances for ``resihp-run --planner module:attr``.

``dp_8mb``: replica-DP with 8 micro-batches (the float64 GPT demo, ``examples/gpt_dp_demo.py``).
``hetero_tp2_pp2_dp2``: the progressive TP -> PP -> DP planner for the reference model of
``examples/hetero_demo.py`` (4 layers, TP2 x PP2 x DP2, sequence parallel, 8 micro-batches).
``gpu_tp2_pp2_dp2``: the same planner for ``GPU_DEMO``, the small Llama-shaped model that
``examples/gpu_hybrid_demo.py`` trains on the GPU runtime (head dim 128, so the tcgen05
attention kernels run it).
"""

from ..models.config import TINY
from ..plan.coordinator_adapter import make_hetero_planner
from ..plan.dp_planner import make_dp_planner
from ..plan.model_spec import ModelProfile, ModelSpec
from ..plan.planner import PlannerConfig

dp_8mb = make_dp_planner(num_microbatches=8)

HETERO_REF = PlannerConfig(
    model=ModelSpec(num_layers=4, hidden=8, ffn=24, num_heads=12, num_kv_heads=12, vocab=16, seq_len=24,
                    micro_batch_size=2),
    profile=ModelProfile(alpha=1e-6, beta=1e-9, last_stage_extra_layers=0.0),
    num_stages=2, num_replicas=2, tp=2, num_microbatches=8, sequence_parallel=True, migration_rounds=16)

hetero_tp2_pp2_dp2 = make_hetero_planner(HETERO_REF)

GPU_DEMO = TINY.with_(name="gpu-demo", hidden=256, heads=2, kv_heads=2, ffn=512, layers=4, vocab_size=512, seq_len=256)
GPU_DEMO_MICRO = 8


def gpu_planner_config(cfg=GPU_DEMO, micro_batch: int = 1, num_microbatches: int = GPU_DEMO_MICRO, tp: int = 2,
                       pp: int = 2, dp: int = 2) -> PlannerConfig:
    spec = ModelSpec(num_layers=cfg.layers, hidden=cfg.hidden, ffn=cfg.ffn, num_heads=cfg.heads,
                     num_kv_heads=cfg.kv_heads, vocab=cfg.vocab_size, seq_len=cfg.seq_len,
                     micro_batch_size=micro_batch)
    return PlannerConfig(model=spec, profile=ModelProfile.b200(spec), num_stages=pp, num_replicas=dp, tp=tp,
                         num_microbatches=num_microbatches, sequence_parallel=True, migration_rounds=16)


gpu_tp2_pp2_dp2 = make_hetero_planner(gpu_planner_config())
