"""Orchestration of the GPU MoE model (expert parallel over 4 gloo ranks with the all-to-all
transport, PyTorch stand-ins for the kernels): gradients of every dense and expert tensor and
the per-step losses must match one rank holding every expert."""

import pytest
import torch

from tests.dist_utils import spawn

pytestmark = pytest.mark.dist


def _cfg():
    from resihp_megatron_b200.models.config import GPTConfig

    return GPTConfig(name="tmoe", vocab_size=64, hidden=64, layers=2, heads=4, kv_heads=2, ffn=64, seq_len=8,
                     num_experts=4, top_k=2)


def _worker(rank, world, port, steps):
    import torch.distributed as dist

    from tests.helpers import fake_kernels

    fake_kernels.install()
    from resihp_megatron_b200.train.moe_trainer import GPUMoETrainer

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    tr = GPUMoETrainer(_cfg(), global_batch=8, micro_batch=1, seq_len=8, ep_impl="collective",
                       dp_impl="collective", device="cpu", lr=1e-2)
    m = tr.model
    # step 0's gradients before any update
    for j in range(tr.n_local):
        ids, labels = tr.tokens.tokens(0, rank * tr.n_local + j)
        m.forward_backward(ids, labels, 1.0 / tr.tokens_per_step)
    dense = m.dense.grad.clone()
    if world > 1:
        dist.all_reduce(dense)
    grads = {n: dense[m.dense.offsets[n]:m.dense.offsets[n] + m.dense.specs[n].numel].clone() for n in m.dense.order}
    grads.update({n: m.experts.g(n).clone() for n in m.experts.order})
    m.dense.grad.zero_()
    m.experts.grad.zero_()
    losses = [tr.train_step() for _ in range(steps)]
    tr.close()
    dist.destroy_process_group()
    return {"grads": grads, "losses": losses}


def test_expert_parallel_moe_matches_one_rank():
    one = spawn(_worker, 1, 2, timeout=240)[0]
    many = spawn(_worker, 4, 2, timeout=300)
    got = {}
    for r in many.values():
        got.update(r["grads"])
    assert set(got) == set(one["grads"])
    for name, want in one["grads"].items():
        err = (got[name] - want).abs().max().item()
        assert err <= 2e-2 * (want.abs().max().item() + 1e-12), (name, err)
    for r, res in many.items():
        for a, b in zip(res["losses"], one["losses"]):
            assert abs(a - b) <= 1e-2 * abs(b), (r, res["losses"], one["losses"])


def _replace(rank, world, port, steps_before, steps_after):
    import torch.distributed as dist

    from tests.helpers import fake_kernels

    fake_kernels.install()
    from resihp_megatron_b200.train.moe_trainer import GPUMoETrainer

    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    tr = GPUMoETrainer(_cfg(), global_batch=8, micro_batch=1, seq_len=8, ep_impl="collective",
                       dp_impl="collective", device="cpu", lr=1e-2)
    losses = [tr.train_step() for _ in range(steps_before)]
    info = None
    if world > 1:
        info = tr.replace_experts({world - 1: 0.5})  # the last rank runs at half speed
    losses += [tr.train_step() for _ in range(steps_after)]
    tr.close()
    dist.destroy_process_group()
    return {"losses": losses, "info": info}


def test_fail_slow_expert_replacement_keeps_the_run():
    ref = spawn(_replace, 1, 4, 0, timeout=240)[0]["losses"]
    res = spawn(_replace, 4, 2, 2, timeout=300)
    holders = res[0]["info"]["holders"]
    assert any(len(h) > 1 for h in holders), holders  # the slow rank's expert got a replica
    for r, out in res.items():
        assert out["info"]["holders"] == holders
        for a, b in zip(out["losses"], ref):
            assert abs(a - b) <= 1e-2 * abs(b), (r, out["losses"], ref)


def _failslow(rank, world, port, steps, slow_rank, slow_from):
    import torch.distributed as dist

    from tests.helpers import fake_kernels

    fake_kernels.install()
    import torch

    from resihp_megatron_b200.models.config import GPTConfig
    from resihp_megatron_b200.train.moe_trainer import GPUMoETrainer

    torch.set_num_threads(1)
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    cfg = GPTConfig(name="tmoe-fs", vocab_size=64, hidden=256, layers=1, heads=4, kv_heads=2, ffn=512, seq_len=64,
                    num_experts=4, top_k=2)
    tr = GPUMoETrainer(cfg, global_batch=8, micro_batch=1, seq_len=64, ep_impl="collective", dp_impl="collective",
                       device="cpu", lr=1e-3)
    tr.enable_failslow(warmup=5, model_ms_per_row=0.01)  # modelled device time: CPU timings are too noisy
    holders0 = [list(h) for h in tr.holders]
    losses = []
    for it in range(steps):
        if rank == slow_rank and it == slow_from:
            tr.set_slowdown(3.0)  # this rank's expert compute now runs 3x slower
        losses.append(tr.train_step())
    out = {"events": tr.failslow_events, "holders0": holders0, "holders": tr.holders, "losses": losses}
    tr.close()
    dist.destroy_process_group()
    return out


def test_fail_slow_rank_is_detected_by_residual_bocd_and_its_experts_replaced():
    """A rank whose expert compute slows 3x from step 14: every rank's per-row expert time (a
    modelled device time with jitter: CPU process timings are far noisier than a GPU's) goes to
    one residual-BOCD detector per rank (median rank = prediction); the slow rank -- and only it --
    is flagged within a few steps on every rank, its experts are re-placed by speed, training
    continues."""
    res = spawn(_failslow, 4, 30, 3, 14, timeout=400)
    firsts = {r: out["events"][0] if out["events"] else None for r, out in res.items()}
    assert all(e is not None for e in firsts.values()), firsts
    ev = firsts[0]
    assert all(e == ev for e in firsts.values())  # every rank decided the same
    assert set(ev["speeds"]) == {3} and ev["speeds"][3] < 0.8, ev
    assert 14 <= ev["iteration"] <= 22, ev
    assert res[0]["holders"] != res[0]["holders0"]
    assert all(abs(l) < 100 for l in res[0]["losses"])
