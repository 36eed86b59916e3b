"""``SpartonHead``: drop-in for hhkbble/sparton's module
(src/sparton/sparton_kernel.py:710-746).

Same constructor ``SpartonHead(vocab_size, hidden_dim, use_bias=False)``, same
``tie_weights(decoder)``, ``load(weights_dict)``, ``init_parameters()`` and
``forward(hidden_states, attention_mask) -> reps[B, V]``.

Keyword-only additions (defaults keep the upstream behaviour):

* ``process_group``: shard the vocabulary over the ranks of a
  ``torch.distributed`` group (NCCL on GPUs). Rank r owns rows
  ``[r*V_s, min(V, (r+1)*V_s))`` of the decoder, ``V_s = ceil(V/n)`` rounded up to
  the kernel's 128-row vocab tile. The forward needs no communication and
  returns ``reps[:, shard]``; the backward all-reduces (sum) the partial
  d_hidden of every rank, in ``grad_reduce_dtype`` (default: fp32 for 16-bit
  inputs, the input dtype otherwise), in chunks of batch rows that overlap
  the remaining backward kernels.
* ``gather_output``: with a process group, all-gather the shards so forward
  returns the full ``reps[B, V]``.
"""
from __future__ import annotations

import math
from typing import Optional

import torch
import torch.distributed as dist
from torch import nn

from . import ops

VOCAB_TILE = 128
# The sharded backward all-reduces d_hidden in chunks of batch rows of about
# this many bytes, each chunk's all-reduce overlapping the next chunk's kernels.
REDUCE_CHUNK_BYTES = 128 << 20
# Opt-in: reduce each chunk as an fp32 reduce-scatter plus an all-gather of
# the parts rounded to the hidden dtype (3/4 of the bytes of the fp32
# all-reduce). Off by default: on 2 B200s with NCCL 2.28 it measured slower
# than NCCL's all-reduce (2.8 vs 2.2 ms for 1 GiB in 8 chunks).
REDUCE_SCATTER_GATHER = False
# How the sharded backward sums the partial d_hidden over the group:
#   "peer": sparton_hidden_allreduce over NVLink peer memory (sparton_b200.peer):
#           only the packed rows (positions before each row's extent, counted on
#           the device) cross NVLink; used when every rank of the group drives a
#           GPU of this node, there are at most 8 of them and the reduction is in
#           fp32; the d_weight / d_bias kernels run on a side stream meanwhile;
#   "nccl": all-reduce of all B*S rows with NCCL, in chunks of batch rows
#           (_HiddenGradReducer), for any group.
HIDDEN_REDUCE = "peer"


def row_chunks(B: int, row_bytes: int, chunk_bytes: Optional[int] = None) -> list:
    """Batch-row ranges [(b0, b1), ...] covering [0, B) in chunks of about
    ``chunk_bytes`` (REDUCE_CHUNK_BYTES by default) of d_hidden, at most 8, as
    even as the rows allow. Depends only on shapes, so every rank takes the same
    collective steps."""
    chunk_bytes = REDUCE_CHUNK_BYTES if chunk_bytes is None else chunk_bytes
    n = max(1, min(B, 8, (B * row_bytes) // max(chunk_bytes, 1)))
    cuts = [B * i // n for i in range(n + 1)]
    return [(a, b) for a, b in zip(cuts, cuts[1:]) if b > a]


class VocabShard:
    """Contiguous vocabulary range owned by one rank."""

    def __init__(self, vocab_size: int, world_size: int, rank: int):
        if world_size < 1 or not 0 <= rank < world_size:
            raise ValueError(f"bad shard spec: world_size={world_size} rank={rank}")
        self.vocab_size = vocab_size
        self.world_size = world_size
        self.rank = rank
        per = -(-vocab_size // world_size)
        self.padded = -(-per // VOCAB_TILE) * VOCAB_TILE if world_size > 1 else vocab_size
        self.start = min(vocab_size, rank * self.padded)
        self.stop = min(vocab_size, self.start + self.padded)

    @property
    def size(self) -> int:
        return self.stop - self.start

    def __repr__(self) -> str:
        return (f"VocabShard(rank={self.rank}/{self.world_size}, "
                f"rows=[{self.start},{self.stop}) of {self.vocab_size})")


class _HiddenGradReducer:
    """Sum over the ranks of the partial d_hidden [B, S, D], chunk by chunk of
    batch rows (``row_chunks``), each chunk reduced as soon as its rows are
    written into ``partial``:

    * with ``REDUCE_SCATTER_GATHER`` set and a reduce dtype wider than
      hidden's (fp32 for 16-bit hidden states, the default): a reduce-scatter
      in the reduce dtype, each rank's part rounded
      once to hidden's dtype, and an all-gather of the rounded parts into the
      result; 3/4 of the bytes of an fp32 all-reduce, with the same rounding
      (fp32 sums, one rounding to the output dtype). The cast and the
      all-gather are issued from a side stream that waits on the
      reduce-scatter, so the compute stream never waits on a collective;
    * otherwise (or when a chunk does not split evenly over the ranks): an
      all-reduce in place.

    ``finish()`` makes the current stream wait for every collective and returns
    d_hidden."""

    def __init__(self, hidden: torch.Tensor, reduce_dtype: torch.dtype, group):
        B, S, D = hidden.shape
        self.group = group
        self.world = dist.get_world_size(group)
        self.out_dtype = hidden.dtype
        self.partial = torch.empty((B, S, D), dtype=reduce_dtype, device=hidden.device)
        self.chunks = row_chunks(B, S * D * self.partial.element_size())
        self.scatter = REDUCE_SCATTER_GATHER and reduce_dtype != hidden.dtype and all(
            ((b1 - b0) * S * D) % self.world == 0 for b0, b1 in self.chunks)
        self.result = (torch.empty((B, S, D), dtype=hidden.dtype, device=hidden.device)
                       if self.scatter else self.partial)
        self.side = None
        if self.scatter and hidden.is_cuda:
            self.side = torch.cuda.Stream(device=hidden.device)
            self.side.wait_stream(torch.cuda.current_stream(hidden.device))
        self.works = []
        self.keep = []  # tensors the collectives in flight read or write

    def reduce(self, b0: int, b1: int) -> None:
        if not self.scatter:
            self.works.append(dist.all_reduce(self.partial[b0:b1], op=dist.ReduceOp.SUM,
                                              group=self.group, async_op=True))
            return
        src = self.partial[b0:b1].reshape(-1)
        # Both buffers come from the current stream's pool: it waits for every
        # collective in finish(), before any later allocation can reuse them.
        part = torch.empty(src.numel() // self.world, dtype=src.dtype, device=src.device)
        low = torch.empty(part.numel(), dtype=self.out_dtype, device=src.device)
        rs = dist.reduce_scatter_tensor(part, src, op=dist.ReduceOp.SUM, group=self.group,
                                        async_op=True)
        if self.side is not None:
            part.record_stream(self.side)
            low.record_stream(self.side)
            with torch.cuda.stream(self.side):
                rs.wait()
                low.copy_(part)
                ag = dist.all_gather_into_tensor(self.result[b0:b1].reshape(-1), low,
                                                 group=self.group, async_op=True)
        else:
            rs.wait()
            low.copy_(part)
            ag = dist.all_gather_into_tensor(self.result[b0:b1].reshape(-1), low,
                                             group=self.group, async_op=True)
        self.keep += [part, low]
        self.works.append(ag)

    def finish(self) -> torch.Tensor:
        for work in self.works:
            work.wait()
        if self.side is not None:
            torch.cuda.current_stream(self.result.device).wait_stream(self.side)
        self.keep.clear()
        return self.result


def _use_peer_reduce(group, hidden, reduce_dtype) -> bool:
    if HIDDEN_REDUCE != "peer" or reduce_dtype != torch.float32:
        return False
    from .peer import PeerHiddenReduce

    return PeerHiddenReduce.usable(group, hidden)


def peer_sharded_backward(grad_reps, reps, idx, hidden, weight, has_bias: bool, need_w: bool,
                          need_b: bool, group, fwd_workspace):
    """Backward of one rank of a vocabulary-sharded head with the d_hidden sum
    over NVLink peer memory: the partial d_hidden into this rank's peer
    buffer, then sparton_hidden_allreduce while the d_weight / d_bias kernels
    run on a side stream. Returns (d_hidden, d_weight or None, d_bias or
    None); every rank takes part, needed or not."""
    from .peer import PeerHiddenReduce

    B, S, D = hidden.shape
    dev = hidden.device
    grad_c = grad_reps.to(hidden.dtype).contiguous()
    reps_c, idx_c = reps.contiguous(), idx.contiguous()
    hidden_c, weight_c = hidden.contiguous(), weight.contiguous()
    peer = PeerHiddenReduce.get(group, dev, B * S, D, hidden.dtype)
    cur = torch.cuda.current_stream(dev)
    # The partial d_hidden first, alone (every rank's reduction waits for all
    # of them); then d_weight / d_bias on a side stream while it is summed.
    ops.hidden_grad_rows(grad_c, reps_c, idx_c, hidden_c, weight_c, peer.partial(B, S), 0, B)
    d_weight = d_bias = None
    side = None
    if need_w or need_b:
        side = torch.cuda.Stream(device=dev)
        side.wait_stream(cur)
        with torch.cuda.stream(side):
            _, d_weight, d_bias = ops.backward_impl(grad_c, reps_c, idx_c, hidden_c, weight_c,
                                                    need_b, need_hidden=False,
                                                    need_embed=need_w)
    d_hidden = torch.empty((B, S, D), dtype=hidden.dtype, device=dev)
    peer.reduce(fwd_workspace, B, S, d_hidden)
    if side is not None:
        cur.wait_stream(side)
        for t in (d_weight, d_bias):
            if t is not None:
                t.record_stream(cur)
    return d_hidden, d_weight, d_bias


class _ShardedHead(torch.autograd.Function):
    """Vocab-sharded head: local fused forward; backward = local gradients plus an
    all-reduce (sum) of the partial d_hidden over the group (HIDDEN_REDUCE)."""

    @staticmethod
    def forward(ctx, hidden, weight, bias, mask, group, reduce_dtype):
        ctx.peer = _use_peer_reduce(group, hidden, reduce_dtype)
        if ctx.peer:
            reps, idx, ctx.fwd_ws = ops.forward_impl(hidden, weight, bias, mask,
                                                     keep_workspace=True)
        else:
            reps, idx = ops.forward_impl(hidden, weight, bias, mask)
        ctx.save_for_backward(reps, idx, hidden, weight)
        ctx.has_bias = bias is not None
        ctx.group = group
        ctx.reduce_dtype = reduce_dtype
        return reps

    @staticmethod
    def backward(ctx, grad_reps):
        reps, idx, hidden, weight = ctx.saved_tensors
        need_h, need_w = ctx.needs_input_grad[0], ctx.needs_input_grad[1]
        need_b = ctx.has_bias and ctx.needs_input_grad[2]
        if ctx.peer:
            d_hidden, d_weight, d_bias = peer_sharded_backward(
                grad_reps, reps, idx, hidden, weight, ctx.has_bias, need_w, need_b, ctx.group,
                ctx.fwd_ws)
            return (d_hidden if need_h else None, d_weight if need_w else None,
                    d_bias if need_b else None, None, None, None)
        # The partial d_hidden first, in chunks of batch rows, each chunk's
        # collectives overlapping the kernels of the next chunk and the last
        # ones the d_weight / d_bias kernels. Every rank takes part in the
        # collectives, whether or not it needs d_hidden.
        reducer = _HiddenGradReducer(hidden, ctx.reduce_dtype, ctx.group)
        grad_c = grad_reps.to(hidden.dtype).contiguous()
        reps_c, idx_c = reps.contiguous(), idx.contiguous()
        hidden_c, weight_c = hidden.contiguous(), weight.contiguous()
        for b0, b1 in reducer.chunks:
            ops.hidden_grad_rows(grad_c, reps_c, idx_c, hidden_c, weight_c, reducer.partial, b0,
                                 b1)
            reducer.reduce(b0, b1)
        d_weight = d_bias = None
        if need_w or need_b:
            _, d_weight, d_bias = ops.backward_impl(
                grad_reps, reps, idx, hidden, weight, need_b, need_hidden=False,
                need_embed=need_w)
        d_hidden = reducer.finish()
        return (d_hidden if need_h else None, d_weight if need_w else None,
                d_bias if need_b else None, None, None, None)


class _GatherVocab(torch.autograd.Function):
    """All-gather of vocab shards [B, V_s] -> [B, V]; backward keeps the local slice."""

    @staticmethod
    def forward(ctx, local, shard: VocabShard, group):
        ctx.shard = shard
        B = local.shape[0]
        buf = local.new_zeros((B, shard.padded))
        buf[:, : local.shape[1]] = local
        parts = [torch.empty_like(buf) for _ in range(shard.world_size)]
        dist.all_gather(parts, buf.contiguous(), group=group)
        return torch.cat(parts, dim=1)[:, : shard.vocab_size].contiguous()

    @staticmethod
    def backward(ctx, grad_full):
        sh = ctx.shard
        return grad_full[:, sh.start:sh.stop].contiguous(), None, None


class SpartonHead(nn.Module):
    """SPLADE head: ``reps[b,v] = max_s log1p(relu((h[b,s]·W[v] + bias[v]) * mask[b,s]))``
    computed by one fused sm_100a kernel (no [B,S,V] logits), with an
    atomic-free fused backward."""

    def __init__(self, vocab_size, hidden_dim, use_bias=False, *,
                 process_group: Optional[dist.ProcessGroup] = None, gather_output: bool = False,
                 grad_reduce_dtype: Optional[torch.dtype] = None):
        super().__init__()
        self.vocab_size = int(vocab_size)
        self.hidden_dim = int(hidden_dim)
        self.process_group = process_group
        self.gather_output = gather_output
        self.grad_reduce_dtype = grad_reduce_dtype
        if process_group is not None:
            world, rank = dist.get_world_size(process_group), dist.get_rank(process_group)
        else:
            world, rank = 1, 0
        self.shard = VocabShard(self.vocab_size, world, rank)
        self.weight = nn.Parameter(torch.empty(self.shard.size, self.hidden_dim))
        if use_bias:
            self.bias = nn.Parameter(torch.empty(self.shard.size))
        else:
            self.register_parameter("bias", None)
        self.init_parameters()

    @property
    def sharded(self) -> bool:
        return self.shard.world_size > 1

    def tie_weights(self, decoder):
        """Alias the decoder's Parameters (upstream :721-723).

        With a process group (vocabulary-sharded) the head's ``weight`` /
        ``bias`` become Parameters over this rank's rows of the decoder's
        tensors: views that share the decoder's storage, so an optimizer step
        on the head writes straight into those rows, while the gradient the
        head accumulates is shard-sized ([V_s, D], not a full [V, D] that is
        zero outside the shard). The decoder's own full Parameters then get no
        gradient from the head, and their rows outside this rank's shard are
        not updated here: ``gather_weights()`` assembles the full, current
        tensors (for a checkpoint, or to refresh the decoder)."""
        if not self.sharded:
            self.weight = decoder.weight
            self.bias = decoder.bias
            return
        sh = self.shard
        if decoder.weight.shape[0] != self.vocab_size:
            raise ValueError(f"decoder has {decoder.weight.shape[0]} rows, head vocab_size "
                             f"{self.vocab_size}")
        self.weight = nn.Parameter(decoder.weight.detach().narrow(0, sh.start, sh.size))
        self.bias = (nn.Parameter(decoder.bias.detach().narrow(0, sh.start, sh.size))
                     if decoder.bias is not None else None)

    @torch.no_grad()
    def gather_weights(self, out_weight: Optional[torch.Tensor] = None,
                       out_bias: Optional[torch.Tensor] = None):
        """(weight [V, D], bias [V] or None): the full parameters assembled from
        every rank's shard (all-gather over the head's group; every rank must
        call it). Unsharded: the head's own tensors. ``out_weight`` /
        ``out_bias`` (e.g. a tied decoder's full Parameters) receive the result
        in place; a checkpoint saved after this holds the trained rows of every
        shard."""
        if not self.sharded:
            w, b = self.weight.detach(), (self.bias.detach() if self.bias is not None else None)
        else:
            w = self._gather_rows(self.weight.detach())
            b = self._gather_rows(self.bias.detach()) if self.bias is not None else None
        if out_weight is not None:
            out_weight.copy_(w)
            w = out_weight
        if out_bias is not None and b is not None:
            out_bias.copy_(b)
            b = out_bias
        return w, b

    def _gather_rows(self, local: torch.Tensor) -> torch.Tensor:
        sh = self.shard
        buf = local.new_zeros((sh.padded,) + tuple(local.shape[1:]))
        buf[: local.shape[0]] = local
        parts = [torch.empty_like(buf) for _ in range(sh.world_size)]
        dist.all_gather(parts, buf.contiguous(), group=self.process_group)
        return torch.cat(parts, dim=0)[: self.vocab_size].contiguous()

    def load(self, weights_dict):
        """Copy ``weights_dict["weight"]`` (and ``["bias"]``) in place (upstream
        :725-734). Full [V, D] tensors are narrowed to this rank's shard."""
        with torch.no_grad():
            self.weight.copy_(self._rows(weights_dict["weight"], self.weight))
            if self.bias is not None and "bias" in weights_dict:
                self.bias.copy_(self._rows(weights_dict["bias"], self.bias))
            else:
                print("no bias")

    def init_parameters(self):
        """nn.Linear's initialisation (upstream :736-741)."""
        nn.init.kaiming_uniform_(self.weight, a=math.sqrt(5))
        if self.bias is not None:
            fan_in = self.hidden_dim
            bound = 1 / math.sqrt(fan_in) if fan_in > 0 else 0
            nn.init.uniform_(self.bias, -bound, bound)

    def _rows(self, full: torch.Tensor, like: torch.Tensor) -> torch.Tensor:
        if self.sharded and full.shape[0] == self.vocab_size and like.shape[0] != self.vocab_size:
            return full[self.shard.start:self.shard.stop]
        return full

    def _local_params(self):
        w, b = self.weight, self.bias
        if self.sharded and w.shape[0] == self.vocab_size and self.shard.size != self.vocab_size:
            w = w.narrow(0, self.shard.start, self.shard.size)
            b = b.narrow(0, self.shard.start, self.shard.size) if b is not None else None
        if b is not None and b.dtype != w.dtype:
            b = b.to(w.dtype)
        return w, b

    def forward(self, hidden_states, attention_mask):
        weight, bias = self._local_params()
        if not (torch.is_grad_enabled() and any(
                t is not None and t.requires_grad for t in (hidden_states, weight, bias))):
            # Nothing will flow back (no_grad / inference_mode, e.g. an encode
            # for indexing): the forward without the argmax output, which
            # skips the [B, V] int32 idx. Same reps. Sharded, no collective is
            # involved either way.
            reps = torch.ops.sparton.fused_sparton_fwd_scores(hidden_states, weight, bias,
                                                             attention_mask)
            if self.sharded and self.gather_output:
                reps = _GatherVocab.apply(reps, self.shard, self.process_group)
            return reps
        if not self.sharded:
            scores, _idx = torch.ops.sparton.fused_sparton_fwd(hidden_states, weight, bias,
                                                               attention_mask)
            return scores
        reduce_dtype = self.grad_reduce_dtype
        if reduce_dtype is None:
            reduce_dtype = (torch.float32 if hidden_states.dtype in (torch.float16, torch.bfloat16)
                            else hidden_states.dtype)
        reps = _ShardedHead.apply(hidden_states, weight, bias, attention_mask,
                                  self.process_group, reduce_dtype)
        if self.gather_output:
            reps = _GatherVocab.apply(reps, self.shard, self.process_group)
        return reps

    def extra_repr(self) -> str:
        return (f"vocab_size={self.vocab_size}, hidden_dim={self.hidden_dim}, "
                f"bias={self.bias is not None}, {self.shard}")
