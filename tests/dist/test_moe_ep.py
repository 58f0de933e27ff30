"""Expert parallelism on gloo ranks, through a rank loss.

Four ranks start as two EP groups of two.  After two iterations the last rank leaves between
steps; the three survivors re-place the experts (sticky, load-aware), move expert weights and
Adam moments with the slice transfer engine, and train on.  Every iteration's loss and every
final tensor must equal single-process float64 training of the same MoE -- with and without the
aux-loss-free routing bias."""

import os

import pytest
import torch

from tests.dist_utils import spawn

pytestmark = pytest.mark.dist

BEFORE, AFTER = 2, 3


def _step(cfg, runtime, optimizer, iteration):
    import torch.distributed as dist

    from resihp_megatron_b200.runtime.moe import batch, token_loss

    optimizer.zero_grad()
    x, y = batch(cfg, iteration)
    lo, hi = runtime.token_range()  # data parallel over tokens
    local = token_loss(runtime.forward(x[lo:hi]), y[lo:hi])
    (local / cfg.tokens).backward()
    runtime.sync_grads()
    optimizer.step()
    runtime.finish_iteration()
    summed = local.detach().reshape(1).clone()
    if runtime.comms.group("dp") is not None:
        runtime.wait(dist.all_reduce(summed, group=runtime.comms.group("dp"), async_op=True))
    return summed.item() / cfg.tokens


def _state_of(params, buffers, optimizer):
    moments = {kind: {k: optimizer.state[k][kind] for k in params} for kind in ("exp_avg", "exp_avg_sq")}
    return {"param": {k: p.data for k, p in params.items()} | buffers, **moments}


def _worker(rank, world, port, store_addr, bias_rate):
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
    everyone = [f"r{i}" for i in range(world)]
    me, prefix = everyone[rank], f"ep{int(100 * bias_rate)}"
    mgr = ResilientCommManager("gloo", timeout_s=30)

    def local_state(placement):
        keys = local_keys(placement, me, specs)
        params = {k: torch.nn.Parameter(init_param(cfg, specs[k])) for k in keys if specs[k].trainable}
        return params, {k: init_param(cfg, specs[k]) for k in keys if not specs[k].trainable}

    first = plan_expert_placement([everyone[:2], everyone[2:]], cfg.num_experts)
    comms = mgr.build(1, everyone, me, moe_group_specs(first, everyone), store_addr=store_addr,
                      store_prefix=f"{prefix}/gen1/")
    params, buffers = local_state(first)
    optimizer = Adam(params, lr=1e-2)
    runtime = EPRuntime(cfg, first, me, everyone, comms, mgr, params, buffers=buffers)
    losses = [_step(cfg, runtime, optimizer, it) for it in range(BEFORE)]
    loads = runtime.global_loads()
    if rank == world - 1:
        os._exit(0)  # leaves between steps, with nothing in flight

    survivors = everyone[:-1]
    second = plan_expert_placement([survivors], cfg.num_experts, loads=loads, prev=first, slots_per_device=3)
    comms = mgr.build(2, survivors, me, moe_group_specs(second, survivors), store_addr=store_addr,
                      store_prefix=f"{prefix}/gen2/")
    old, new = moe_holdings(first, specs), moe_holdings(second, specs)
    moves = plan_transfers(old, new, valid_sources=set(survivors), node_of=dict.fromkeys(everyone, "n0"))
    assert not moves.lost
    moved = execute_transfers(moves, me, comms, mgr, specs=specs, old_layout=device_layout(old, me),
                              old_state=_state_of(params, buffers, optimizer), new_layout=device_layout(new, me),
                              kinds=("param", "exp_avg", "exp_avg_sq"), dtype=cfg.dtype, timeout=30)
    keys = local_keys(second, me, specs)
    params2 = {k: torch.nn.Parameter(moved["param"][k].clone()) for k in keys if specs[k].trainable}
    buffers2 = {k: moved["param"][k].clone() for k in keys if not specs[k].trainable}
    optimizer2 = Adam(params2, lr=1e-2)
    restored = {f"param/{k}": v for k, v in params2.items()}
    for kind in ("exp_avg", "exp_avg_sq"):
        restored |= {f"{kind}/{k}": moved[kind][k] for k in params2}
    optimizer2.load_state_tensors(restored, optimizer.step_count)
    runtime = EPRuntime(cfg, second, me, survivors, comms, mgr, params2, buffers=buffers2)
    losses += [_step(cfg, runtime, optimizer2, it) for it in range(BEFORE, BEFORE + AFTER)]
    result = {"losses": losses, "final": {k: v.detach().clone() for k, v in params2.items()} | buffers2,
              "moved": moved_experts(first, second), "received": sum(t.dst == me for t in moves.transfers)}
    mgr.destroy()
    return result


@pytest.mark.parametrize("bias_rate", [0.0, 0.05])
def test_rank_loss_re_places_experts_and_training_stays_exact(store, bias_rate):
    from resihp_megatron_b200.runtime.moe import MoEConfig, reference_train

    results = spawn(_worker, 4, store, bias_rate, timeout=240, expect_dead={3})
    assert sorted(results) == [0, 1, 2]
    cfg = MoEConfig(bias_update_rate=bias_rate)
    want_losses, want_final = reference_train(cfg, BEFORE + AFTER)
    for res in results.values():
        assert res["losses"] == pytest.approx(want_losses, rel=1e-10)
        for key, value in res["final"].items():
            torch.testing.assert_close(value, want_final[key], rtol=1e-10, atol=1e-12)
    if bias_rate:  # the routing bias moved, and it travelled with the re-placement
        assert want_final["router.expert_bias"].abs().sum() > 0
        assert all("router.expert_bias" in r["final"] for r in results.values())
    assert results[0]["moved"] > 0 and sum(r["received"] for r in results.values()) > 0
