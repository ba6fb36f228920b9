"""Multi-GPU sampling over torch.distributed (one process per GPU).

Row-sharded mode needs nothing here: each rank samples its own rows with
mxs_sampler.sample() and no collective (rows are independent).

Vocab-sharded mode (VocabShardedSampler): every rank holds the same rows but
only its own column shard [rank*C, (rank+1)*C) of the vocabulary.
  1. each rank lists, per row, every logit of its shard >= the shard's k-th
     largest value (mxs_shard_candidates; ties kept);
  2. one all-gather brings every shard's lists to every rank;
  3. every rank merges them and draws (mxs_merge_sample) - the same inputs on
     every rank give the same result on every rank;
  4. rows whose merged lists show a tie are handed back: the reference's tie
     order depends on every logit of the row, so their full rows are gathered
     (a second all-gather, only when such rows exist) and sampled whole.
The union of the shards' lists holds every logit >= the row's k-th largest
value, because a shard's k-th largest never exceeds the row's.

The kernel-side calls are injectable (shard_fn, merge_fn, full_fn) so the
collective logic can be exercised on CPU ranks with the gloo backend.
"""
import torch
import torch.distributed as dist

from . import ROW_EXACT, k_use, merge_sample, sample, shard_candidates


def _all_gather(t, group):
    """[world, *t.shape] gathered along a new leading dimension."""
    world = dist.get_world_size(group)
    out = torch.empty((world,) + tuple(t.shape), dtype=t.dtype, device=t.device)
    try:
        dist.all_gather_into_tensor(out, t.contiguous(), group=group)
    except (RuntimeError, NotImplementedError, AttributeError):
        dist.all_gather(list(out.unbind(0)), t.contiguous(), group=group)
    return out


class VocabShardedSampler:
    def __init__(self, vocab, group=None, cap=None, shard_fn=None, merge_fn=None, full_fn=None):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.vocab = int(vocab)
        if self.vocab % self.world:
            raise ValueError("vocab must split evenly across the ranks")
        self.cols = self.vocab // self.world
        self.col_offset = self.rank * self.cols
        self.cap = cap
        self.shard_fn = shard_fn or shard_candidates
        self.merge_fn = merge_fn or merge_sample
        self.full_fn = full_fn or (lambda rows, T, k, u, top_p, min_p: sample(rows, T, k, u, top_p, min_p))

    def sample(self, shard_logits, temperature, top_k, u, top_p=1.0, min_p=0.0):
        """shard_logits: [rows, vocab / world] (this rank's columns). u: [rows]
        float64 uniforms, identical on every rank. Returns (next, topk_idx,
        topk_prob, row_flags) for all rows, identical on every rank."""
        rows, cols = shard_logits.shape
        if cols != self.cols:
            raise ValueError(f"expected {self.cols} columns per shard, got {cols}")
        k = k_use(int(top_k), self.vocab)
        cap = self.cap or (2 * min(k, cols) + 64)
        cand, cnt, flg = self.shard_fn(shard_logits, self.col_offset, top_k, cap)
        cand_all = _all_gather(cand, self.group)
        cnt_all = _all_gather(cnt, self.group)
        flg_all = _all_gather(flg, self.group)
        nxt, idx, prob, rflags = self.merge_fn(cand_all, cnt_all, flg_all, self.vocab, temperature, top_k, u,
                                               top_p, min_p)
        redo = torch.nonzero((rflags & ROW_EXACT) != 0).flatten()
        if redo.numel():
            # full rows of the tied rows: gather every rank's columns of them
            parts = _all_gather(shard_logits.index_select(0, redo), self.group)
            full = parts.permute(1, 0, 2).reshape(redo.numel(), self.vocab).contiguous()
            n2, i2, p2 = self.full_fn(full, temperature, top_k, u.index_select(0, redo).contiguous(), top_p, min_p)
            nxt[redo] = n2
            idx[redo] = i2
            prob[redo] = p2
        return nxt, idx, prob, rflags
