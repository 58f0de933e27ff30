"""The MoE decoder (``models.moe_model``) on one GPU: the peer-memory expert transport (router,
dispatch, combine and gradient kernels, one routing state per layer) must train like the
all-to-all transport on the same kernels and weights."""

import math

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_peer_and_collective_expert_transport_agree():
    import torch.distributed as dist

    from resihp_megatron_b200 import ops
    from resihp_megatron_b200.models.config import GPTConfig
    from resihp_megatron_b200.train.hybrid_trainer import ensure_process_group
    from resihp_megatron_b200.train.moe_trainer import GPUMoETrainer

    cfg = GPTConfig(name="tmoe", vocab_size=512, hidden=256, layers=2, heads=2, kv_heads=1, ffn=512, seq_len=256,
                    num_experts=4, top_k=2)
    ensure_process_group(torch.device("cuda", torch.cuda.current_device()))
    try:
        runs = {}
        for impl in ("peer", "collective"):
            tr = GPUMoETrainer(cfg, global_batch=2, micro_batch=1, seq_len=256, ep_impl=impl, dp_impl="collective",
                               lr=3e-3)
            l0 = ops.launches()
            runs[impl] = [tr.train_step() for _ in range(3)]
            assert ops.launches() > l0
            tr.close()
        for a, b in zip(runs["peer"], runs["collective"]):
            assert math.isfinite(a) and abs(a - b) <= 2e-2 * abs(b), runs
        assert abs(runs["peer"][0] - math.log(cfg.vocab_size)) < 0.5
    finally:
        dist.destroy_process_group()
