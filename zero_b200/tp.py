"""Tensor-parallel host plumbing for the Qwen3 decode.

One process per GPU.  Each rank builds its slice of the model
(Qwen3Model(..., rank=r, world=N)); the ranks then swap the CUDA IPC handles
of their activation vectors over any torch.distributed group (gloo or nccl)
and map each other's vectors, after which every rank's persistent step kernel
stores its stage outputs straight into all ranks' copies over NVLink.

The split follows the reference's SMP row partition (smp_partition.rs:108-183:
whole 4-row groups per worker), spread over GPUs instead of cores:

  q / k / v      the q heads and kv heads of kv-head group r (attention and
                 the KV cache stay on the rank)
  O, down        hidden rows [r H/N, (r+1) H/N)
  gate / up      SwiGLU units [r F/4N, (r+1) F/4N), i.e. act rows [r F/N, ...)
  LM head        vocabulary rows [r V/N, (r+1) V/N); the argmax is merged
                 across ranks (larger logit, smaller row on ties)

Every output row is reduced exactly as on one GPU, so a tensor-parallel
decode gives the one-GPU tokens and logits bit for bit.
"""
from __future__ import annotations

from dataclasses import dataclass


@dataclass(frozen=True)
class Slice:
    start: int
    stop: int

    @property
    def size(self) -> int:
        return self.stop - self.start


def check_shardable(cfg, world: int) -> None:
    """The divisibility zgpu_qwen3_create_tp requires (ValueError if not met)."""
    if not 1 <= world <= 8:
        raise ValueError("tensor parallel: 1..8 ranks")
    lm_unit = 8 if cfg.output_quant == "q4_0" else 4
    if world > 1 and (cfg.n_kv_heads % world or cfg.hidden % (8 * world) or cfg.ffn % (8 * world)
                      or cfg.vocab_padded % (lm_unit * world)):
        raise ValueError(f"{cfg.name}: kv heads, hidden / 8, ffn / 8 and LM-head units must divide by {world}")


def shard_plan(cfg, world: int) -> list[dict[str, Slice]]:
    """Per rank: the rows it owns in each output vector."""
    check_shardable(cfg, world)
    out = []
    qd, kvd = cfg.q_dim // world, cfg.kv_dim // world
    H, F, V = cfg.hidden // world, cfg.ffn // world, cfg.vocab_padded // world
    for r in range(world):
        out.append({
            "q": Slice(r * qd, (r + 1) * qd),
            "kv": Slice(r * kvd, (r + 1) * kvd),
            "hidden": Slice(r * H, (r + 1) * H),
            "act": Slice(r * F, (r + 1) * F),
            "vocab": Slice(r * V, (r + 1) * V),
        })
    return out


def expert_plan(n_experts: int, world: int) -> list[Slice]:
    """Expert parallelism (the DeepSeek2 MoE layers): rank r runs routed
    experts [r E/N, (r+1) E/N), the split zgpu_ds2_create_ep makes; the
    router, attention, dense layers, shared experts and LM head run on every
    rank.  ValueError where the C side refuses the split."""
    if not 1 <= world <= 8:
        raise ValueError("expert parallel: 1..8 ranks")
    if n_experts == 0 or n_experts % world:
        raise ValueError(f"expert parallel: {n_experts} experts do not split over {world} ranks")
    per = n_experts // world
    return [Slice(r * per, (r + 1) * per) for r in range(world)]


def expert_owner(expert: int, n_experts: int, world: int) -> int:
    """The rank that runs `expert` and publishes its output row."""
    return expert // (n_experts // world)


def exchange_handles(handle: bytes, group=None) -> list[bytes]:
    """All ranks' handles in rank order (torch.distributed all_gather_object)."""
    import torch.distributed as dist

    world = dist.get_world_size(group)
    got: list = [None] * world
    dist.all_gather_object(got, handle, group=group)
    return [bytes(h) for h in got]


def connect(model, group=None) -> None:
    """Export this rank's handle, gather everyone's, map the peers, then wait
    until every rank has mapped them.  The device-side waits for a peer are
    bounded, so no rank may start its first exchange while another is still
    opening handles (the first peer mapping of a process can take long)."""
    import torch.distributed as dist

    model.tp_connect(exchange_handles(model.tp_export(), group))
    dist.barrier(group=group)
