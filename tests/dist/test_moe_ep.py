"""Expert parallelism over gloo ranks: two EP groups of two, then one rank leaves between steps;
the survivors re-place the experts (sticky, speed-aware), move expert parameters and Adam state
with the transfer engine, and keep training.  Losses and parameters must match the
single-process float64 MoE reference for every iteration, before and after the loss."""

import os

import pytest
import torch

from tests.dist_utils import spawn

pytestmark = pytest.mark.dist

ITERS_BEFORE, ITERS_AFTER = 2, 3


def _train(cfg, rt, opt, it):
    import torch.distributed as dist

    from resihp_megatron_b200.runtime.moe import batch, token_loss

    opt.zero_grad()
    x, y = batch(cfg, it)
    a, b = rt.token_range()
    loss = token_loss(rt.forward(x[a:b]), y[a:b])
    (loss / cfg.tokens).backward()
    rt.sync_grads()
    opt.step()
    rt.finish_iteration()
    total = loss.detach().reshape(1).clone()
    group = rt.comms.group("dp")
    if group is not None:
        rt.wait(dist.all_reduce(total, group=group, async_op=True))
    return total.item() / cfg.tokens


def _ep(rank, world, port, store_addr, bias_rate):
    from resihp_megatron_b200.comm.comm_manager import ResilientCommManager
    from resihp_megatron_b200.plan.expert_placement import moved_experts, plan_expert_placement
    from resihp_megatron_b200.runtime.moe import (EPRuntime, MoEConfig, init_param, local_keys, moe_group_specs,
                                                  moe_holdings, moe_specs)
    from resihp_megatron_b200.runtime.optim import Adam
    from resihp_megatron_b200.state.layer_registry import device_layout
    from resihp_megatron_b200.state.transfer_engine import execute_transfers
    from resihp_megatron_b200.state.transfer_plan import plan_transfers

    cfg = MoEConfig(bias_update_rate=bias_rate)
    specs = moe_specs(cfg)
    ids = [f"w{i}" for i in range(world)]
    me = ids[rank]
    tag = f"moe{int(bias_rate * 100)}"
    mgr = ResilientCommManager("gloo", timeout_s=30)
    p1 = plan_expert_placement([ids[:2], ids[2:]], cfg.num_experts)
    comms = mgr.build(1, ids, me, moe_group_specs(p1, ids), store_addr=store_addr, store_prefix=f"{tag}/gen1/")
    keys = local_keys(p1, me, specs)
    params = {k: torch.nn.Parameter(init_param(cfg, specs[k])) for k in keys if specs[k].trainable}
    buffers = {k: init_param(cfg, specs[k]) for k in keys if not specs[k].trainable}
    opt = Adam(params, lr=1e-2)
    rt = EPRuntime(cfg, p1, me, ids, comms, mgr, params, buffers=buffers)
    losses = [_train(cfg, rt, opt, it) for it in range(ITERS_BEFORE)]
    loads = rt.global_loads()
    if rank == world - 1:
        os._exit(0)  # leaves between steps: nothing of it is in flight
    # survivors: a new generation, sticky re-placement on three devices, state moved
    survivors = ids[:-1]
    p2 = plan_expert_placement([survivors], cfg.num_experts, loads=loads, prev=p1, slots_per_device=3)
    comms2 = mgr.build(2, survivors, me, moe_group_specs(p2, survivors), store_addr=store_addr,
                       store_prefix=f"{tag}/gen2/")
    old_h, new_h = moe_holdings(p1, specs), moe_holdings(p2, specs)
    xfer = plan_transfers(old_h, new_h, valid_sources=set(survivors), node_of={d: "n0" for d in ids})
    assert not xfer.lost
    kinds = ("param", "exp_avg", "exp_avg_sq")
    old_state = {"param": {**{k: p.data for k, p in params.items()}, **buffers},
                 "exp_avg": {k: opt.state[k]["exp_avg"] for k in params},
                 "exp_avg_sq": {k: opt.state[k]["exp_avg_sq"] for k in params}}
    new_state = execute_transfers(xfer, me, comms2, mgr, specs=specs, old_layout=device_layout(old_h, me),
                                  old_state=old_state, new_layout=device_layout(new_h, me), kinds=kinds,
                                  dtype=cfg.dtype, timeout=30)
    keys2 = local_keys(p2, me, specs)
    params2 = {k: torch.nn.Parameter(new_state["param"][k].clone()) for k in keys2 if specs[k].trainable}
    buffers2 = {k: new_state["param"][k].clone() for k in keys2 if not specs[k].trainable}
    opt2 = Adam(params2, lr=1e-2)
    opt2.load_state_tensors({**{f"param/{k}": v for k, v in params2.items()},
                             **{f"exp_avg/{k}": new_state["exp_avg"][k] for k in params2},
                             **{f"exp_avg_sq/{k}": new_state["exp_avg_sq"][k] for k in params2}}, opt.step_count)
    rt2 = EPRuntime(cfg, p2, me, survivors, comms2, mgr, params2, buffers=buffers2)
    losses += [_train(cfg, rt2, opt2, it) for it in range(ITERS_BEFORE, ITERS_BEFORE + ITERS_AFTER)]
    out = {"losses": losses, "params": {k: v.detach().clone() for k, v in params2.items()} | buffers2,
           "replicated": any(len(p2.group_holders(0, e)) > 1 for e in range(cfg.num_experts)),
           "moved": moved_experts(p1, p2), "received": sum(1 for t in xfer.transfers if t.dst == me)}
    mgr.destroy()
    return out


@pytest.mark.parametrize("bias_rate", [0.0, 0.05])
def test_ep_rank_loss_replaces_experts_and_training_matches_reference(store, bias_rate):
    from resihp_megatron_b200.runtime.moe import MoEConfig, reference_train

    out = spawn(_ep, 4, store, bias_rate, timeout=240, expect_dead={3})
    alive = [out[r] for r in sorted(out)]
    assert len(alive) == 3
    cfg = MoEConfig(bias_update_rate=bias_rate)
    ref_losses, ref_params = reference_train(cfg, ITERS_BEFORE + ITERS_AFTER)
    for r in alive:
        assert r["losses"] == pytest.approx(ref_losses, rel=1e-10)
        for k, v in r["params"].items():
            torch.testing.assert_close(v, ref_params[k], rtol=1e-10, atol=1e-12)
    if bias_rate:
        assert ref_params["router.expert_bias"].abs().sum() > 0
        assert all("router.expert_bias" in r["params"] for r in alive)
    assert alive[0]["moved"] > 0 and sum(r["received"] for r in alive) > 0
