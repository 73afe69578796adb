"""Speculative decoding: n-gram or draft-model proposals verified by one
target forward per step.

Each step:
  1. every running sequence that is ready for a plain decode gets up to k
     draft tokens (k adapts to the measured acceptance rate), appended to it
     in the C++ core (``Scheduler.append_tokens``);
  2. the scheduler builds the batch as usual; a drafted sequence computes
     its last real token plus the drafts (query length 1 + k) through the
     paged prefill kernel, and its logits are taken at all 1 + k positions;
  3. verification on the device: greedy requests accept the longest prefix of
     drafts equal to the target's argmax; sampled requests use rejection
     sampling (accept draft d with probability min(1, p(d) / q(d)), on
     rejection draw from normalise(max(p - q, 0)); an n-gram draft has q =
     one-hot), so the output follows the target's own sampling distribution;
     the token after the last accepted draft is the target's (the "bonus"
     token when every draft is accepted);
  4. the drafts are rolled back and the verified tokens appended with the
     stop rules applied per token (``Scheduler.update_multi``), keeping the
     KV the verification step wrote for them.

Requests with penalties, logprobs or stop strings are not drafted (they take
one token per step inside the same batches).

Draft model: a second, smaller decoder with the same vocabulary runs on the
engine's own GPU. Its KV pool has the same number of blocks as the target's
and uses the SAME block tables and slot mapping, so the block manager needs
no second bookkeeping; it also runs every target step's batch, which keeps
its KV for prompts and verified tokens current.

Parity: crates/swiftllm-core/src/execution/speculative.rs (SpeculativeDecoder
:49-255 with verify :97-167, adjusted distribution :170-190, adaptive k
:214-231; NgramSpeculator :294-372). There the verifier is a CPU library
that the engine never calls; here it is wired into the engine step.
"""

from __future__ import annotations

import time
from typing import Dict, List, Optional

import numpy as np
import torch

from .. import _core
from ..outputs import RequestOutput
from ..utils.logging import get_logger

log = get_logger(__name__)

NGRAM_NAMES = ("ngram", "[ngram]")


def is_ngram(name: Optional[str]) -> bool:
    return bool(name) and name.lower() in NGRAM_NAMES


def reserve_draft_memory(cfg) -> None:
    """Tell the target's KV sizing how much to leave for a draft model:
    its weights and, per KV block, the draft's own KV block."""
    if not cfg.speculative_model or is_ngram(cfg.speculative_model):
        return
    from ..models.config import load_config
    from ..models.decoder import DecoderModel
    dc = load_config(cfg.speculative_model)
    el = 4 if getattr(cfg.dtype, "value", cfg.dtype) == "float32" else 2
    cfg.draft_block_bytes = dc.num_layers * 2 * dc.num_kv_heads * cfg.block_size * dc.head_dim * el
    m = DecoderModel(dc, torch.bfloat16, "meta")
    m.allocate()
    cfg.draft_reserve_bytes = sum(p.numel() for _, p in m.named_parameters()) * el


def processed_probs(logits: torch.Tensor, temp: torch.Tensor, top_k: torch.Tensor,
                    top_p: torch.Tensor, min_p: torch.Tensor) -> torch.Tensor:
    """Sampling distribution of each row: temperature -> min-p -> top-k (ties
    kept) -> top-p (the token that crosses the mass is kept), renormalised.
    Same order as the fused sampling kernel."""
    x = logits.float() / temp.clamp_min(1e-6).unsqueeze(1)
    p = torch.softmax(x, dim=-1)
    V = p.shape[1]
    keep = p >= (min_p.unsqueeze(1) * p.amax(1, keepdim=True))
    k = torch.where(top_k > 0, top_k.clamp(max=V), torch.full_like(top_k, V)).long()
    sp, _ = p.sort(dim=-1, descending=True)
    kth = sp.gather(1, (k - 1).unsqueeze(1))
    keep &= p >= kth
    p = torch.where(keep, p, torch.zeros_like(p))
    p = p / p.sum(1, keepdim=True)
    sp, si = p.sort(dim=-1, descending=True)
    before = sp.cumsum(1) - sp
    drop_sorted = before >= top_p.unsqueeze(1)
    drop = torch.zeros_like(drop_sorted).scatter(1, si, drop_sorted)
    p = torch.where(drop, torch.zeros_like(p), p)
    return p / p.sum(1, keepdim=True)


class SpeculativeDecoder:
    def __init__(self, engine, spec_model: str, num_tokens: int, ngram_n: int = 3):
        self.engine = engine
        self.k_max = max(1, int(num_tokens))
        self.adaptive = _core.AdaptiveK(self.k_max, 1, self.k_max, 0.6)
        self.ngram = None
        self.draft = None
        dev = engine.executor.device
        self.device = dev
        self.gen = torch.Generator(device=dev)
        self.gen.manual_seed(int(engine.config.seed) * 7919 + 17)
        if is_ngram(spec_model):
            self.ngram = _core.NgramSpeculator(ngram_n, self.k_max)
        else:
            self._init_draft(spec_model)
        self.stats = {"steps": 0, "proposed": 0, "accepted": 0, "emitted": 0}

    # ------------------------------------------------------------ draft model
    def _init_draft(self, name: str) -> None:
        import copy
        from ..models.config import load_config
        from ..runtime.model_runner import ModelRunner
        e = self.engine
        dcfg = load_config(name)
        if dcfg.vocab_size != e.model_config.vocab_size:
            raise ValueError(f"draft model vocab {dcfg.vocab_size} != target vocab "
                             f"{e.model_config.vocab_size}")
        ec = copy.copy(e.config)
        ec.model = name
        ec.load_format = "dummy" if e.config.load_format == "dummy" else "auto"
        self.draft = ModelRunner(dcfg, ec, self.device, max_model_len=e.config.max_model_len)
        self.draft.load_weights()
        self.draft.allocate_kv(e.executor.num_gpu_blocks, 0)
        if self.draft.use_graphs:
            self.draft.capture_graphs(min(e.config.max_num_seqs, 256))

    def _decode_input(self, toks: np.ndarray, pos: np.ndarray, slots: np.ndarray,
                      tables: np.ndarray):
        from ..runtime.model_runner import StepInput
        S = toks.shape[0]
        MB = tables.shape[1]
        ints = np.concatenate([toks, pos, slots, np.arange(S + 1, dtype=np.int32), pos + 1,
                               tables.reshape(-1)]).astype(np.int32)
        e2 = np.zeros((0, 2), np.int64)
        return StepInput(S, S, S, 1, int(pos.max()) + 1, MB, ints, np.arange(S, dtype=np.int32),
                         e2, e2, e2)

    def _propose_draft(self, sids: List[int], ks: List[int], params: List) -> Dict[int, tuple]:
        """k autoregressive draft steps for all sequences at once. Returns
        sid -> (draft tokens, q rows [k, V] on the device or None for greedy)."""
        e = self.engine
        sch, bm = e.scheduler, e.block_manager
        bs = e.config.block_size
        S, K = len(sids), max(ks)
        tabs = [np.asarray(bm.get_block_table(s), dtype=np.int32) for s in sids]
        MB = max(len(t) for t in tabs)
        tables = np.full((S, MB), -1, dtype=np.int32)
        for i, t in enumerate(tabs):
            tables[i, :len(t)] = t
        L = np.array([sch.seq_info(s)["num_tokens"] for s in sids], dtype=np.int32)
        cur = np.array([int(sch.seq_tokens(s, False)[-1]) for s in sids], dtype=np.int32)
        greedy = np.array([p.temperature == 0 or p.top_k == 1 for p in params])
        dev = self.device
        if not greedy.all():
            pt = torch.tensor([max(p.temperature, 1e-6) for p in params], device=dev)
            pk = torch.tensor([p.top_k for p in params], device=dev)
            pp = torch.tensor([p.top_p for p in params], device=dev)
            pm = torch.tensor([p.min_p for p in params], device=dev)
        drafts = np.zeros((S, K), dtype=np.int32)
        qs = []
        kk = np.asarray(ks)
        for j in range(K):
            pos = (L - 1 + j).astype(np.int32)
            live = j < kk
            blk = np.where(live, tables[np.arange(S), np.minimum(pos // bs, MB - 1)], -1)
            slots = np.where(live & (blk >= 0), blk * bs + pos % bs, -1).astype(np.int32)
            logits = self.draft.execute(self._decode_input(cur, pos, slots, tables))
            nxt = logits.argmax(-1)
            if not greedy.all():
                q = processed_probs(logits, pt, pk, pp, pm)
                samp = torch.multinomial(q, 1, generator=self.gen).view(-1)
                g = torch.from_numpy(greedy).to(dev)
                nxt = torch.where(g, nxt, samp)
                qs.append(q)
            cur = nxt.to(torch.int32).cpu().numpy()
            drafts[:, j] = cur
        out = {}
        for i, s in enumerate(sids):
            qrows = None if greedy[i] else torch.stack([qs[j][i] for j in range(ks[i])])
            out[s] = (drafts[i, :ks[i]].tolist(), qrows)
        return out

    # ------------------------------------------------------------ step
    def _eligible(self, sid: int):
        e = self.engine
        info = e.scheduler.seq_info(sid)
        r = e._by_gid.get(int(info["group"]))
        if r is None:
            return None
        sp = r.params
        if sp.logprobs is not None or sp.stop or sp.presence_penalty or sp.frequency_penalty \
                or sp.repetition_penalty != 1.0:
            return None
        L = int(info["num_tokens"])
        k = min(self.adaptive.k, sp.max_tokens - int(info["num_output"]) - 1,
                e.config.max_model_len - L - 1)
        if self.draft is not None:
            # the draft writes KV for positions L-1 .. L+k-2 before the
            # scheduler grows the table: stay inside the reserved slots
            cap = len(e.block_manager.get_block_table(sid)) * e.config.block_size
            k = min(k, cap - L + 1)
        return (r, k) if k > 0 else None

    def step(self) -> List[RequestOutput]:
        from ..runtime.model_runner import step_input_from_batch
        e = self.engine
        sch = e.scheduler
        self.stats["steps"] += 1
        # 1. proposals
        drafted: Dict[int, tuple] = {}
        cands = []
        for sid in sch.decode_ready_seqs().tolist():
            el = self._eligible(int(sid))
            if el is not None:
                cands.append((int(sid), el[0], el[1]))
        if self.ngram is not None:
            for sid, r, k in cands:
                d = self.ngram.propose(sch.seq_tokens(sid, False), k)
                if len(d):
                    drafted[sid] = (list(map(int, d))[:k], None)
        elif cands:
            drafted = self._propose_draft([c[0] for c in cands], [c[2] for c in cands],
                                          [c[1].params for c in cands])
        for sid, (d, _) in drafted.items():
            sch.append_tokens(sid, d)
        # 2. schedule + target forward over 1 + k positions of drafted rows
        b = sch.schedule(time.monotonic())
        outs = e._rejected(b)
        if b.num_seqs == 0 and b.swap_in.size == 0 and b.swap_out.size == 0:
            self._rollback(drafted)
            return outs
        si = step_input_from_batch(b)
        q_start = np.asarray(b.q_start)
        q_len = np.asarray(b.q_len)
        seq_ids = np.asarray(b.seq_ids)
        srow = np.asarray(b.sample_seq_row)
        lrows = np.asarray(b.sample_logit_idx)
        nl = si.logits_idx.shape[0]
        row_of_l = np.zeros(nl, dtype=np.int64)
        row_of_l[lrows] = srow
        kl = np.zeros(nl, dtype=np.int64)
        for l in range(nl):
            d = drafted.get(int(seq_ids[row_of_l[l]]))
            if d is not None and q_len[row_of_l[l]] == len(d[0]) + 1:
                kl[l] = len(d[0])
        first = (q_start[:-1][row_of_l] + q_len[row_of_l] - 1 - kl).astype(np.int64)
        base = np.concatenate([[0], np.cumsum(kl + 1)]).astype(np.int64)
        new_idx = np.concatenate([np.arange(f, f + k + 1) for f, k in zip(first, kl)]) \
            if nl else np.zeros(0, np.int64)
        si.logits_idx = new_idx.astype(np.int32)
        if self.draft is not None:
            self.draft.execute(si)  # keeps the draft's KV current (same slots)
        logits = e.executor.execute(si)
        if b.num_sample_rows == 0:
            self._rollback(drafted)
            e._account(si, b, 0)
            return outs
        dev = logits.device
        last = torch.from_numpy(base[1:] - 1).to(dev)
        logits_last = logits.index_select(0, last)
        toks, lps = e.sampler(logits_last, b, e._history)
        want_lp = e._top_logprobs(logits_last, b, toks) if e._wants_logprobs(b) else None
        # 3. verification of every draft position
        nrows = int(b.num_sample_rows)
        temp = np.asarray(b.temperature, dtype=np.float32)
        topk = np.asarray(b.top_k, dtype=np.int32)
        counts = np.ones(nrows, dtype=np.int32)
        vpos, vdraft, vrow = [], [], []
        for r in range(nrows):
            l = lrows[r]
            if kl[l] == 0:
                continue
            d = drafted[int(seq_ids[srow[r]])][0]
            vpos.extend(range(base[l], base[l] + kl[l]))
            vdraft.extend(d)
            vrow.extend([r] * len(d))
        flat_t: List[int] = []
        flat_lp: List[float] = []
        if vpos:
            acc, alt, lp_d, lp_a = self._verify(logits, b, drafted, np.asarray(vpos),
                                                np.asarray(vdraft, np.int64), np.asarray(vrow),
                                                temp, topk)
        j = 0
        for r in range(nrows):
            l = lrows[r]
            k = int(kl[l])
            if k == 0:
                flat_t.append(int(toks[r]))
                flat_lp.append(float(lps[r]))
                continue
            a = 0
            while a < k and acc[j + a]:
                a += 1
            d = drafted[int(seq_ids[srow[r]])][0]
            flat_t.extend(d[:a])
            flat_lp.extend(lp_d[j:j + a].tolist())
            if a < k:
                flat_t.append(int(alt[j + a]))
                flat_lp.append(float(lp_a[j + a]))
            else:
                flat_t.append(int(toks[r]))
                flat_lp.append(float(lps[r]))
            counts[r] = a + 1
            self.adaptive.update(k, a)
            self.stats["proposed"] += k
            self.stats["accepted"] += a
            j += k
        # 4. roll back drafts, append verified tokens
        self._rollback(drafted)
        res = sch.update_multi(b, np.asarray(flat_t, np.int32), counts,
                               np.asarray(flat_lp, np.float32), time.monotonic())
        e._gen_tokens += len(res.token)
        self.stats["emitted"] += len(res.token)
        e._account(si, b, len(res.token))
        return outs + e._process(res, want_lp)

    def _rollback(self, drafted) -> None:
        sch = self.engine.scheduler
        for sid, (d, _) in drafted.items():
            info = sch.seq_info(sid)
            if info is not None and d:
                sch.rollback(sid, len(d))

    def _verify(self, logits, b, drafted, vpos, vdraft, vrow, temp, topk):
        """-> accepted [M] bool, replacement token [M], logprob of the draft
        [M], logprob of the replacement [M] (host arrays)."""
        dev = logits.device
        pos = torch.from_numpy(vpos).to(dev)
        d = torch.from_numpy(vdraft).to(dev)
        greedy = (temp[vrow] == 0) | (topk[vrow] == 1)
        t = torch.from_numpy(np.where(temp[vrow] > 0, temp[vrow], 1.0).astype(np.float32)).to(dev)
        if greedy.all() and logits.is_cuda and logits.dtype == torch.float32:
            # one kernel: arg-max, log-sum-exp and both log-probabilities per position
            from .. import ops
            out = torch.empty(4, len(vpos), dtype=torch.float32, device=dev)
            ops.cuda_ext().spec_verify_greedy(logits, pos, d, t, out)
            ops._count()
            both = out.cpu().numpy()
            return both[0] > 0.5, both[1].astype(np.int64), both[2], both[3]
        x = logits.index_select(0, pos).float()
        lsm = torch.log_softmax(x / t.unsqueeze(1), dim=-1)
        am = x.argmax(-1)
        acc = am == d
        alt = am.clone()
        if not greedy.all():
            rnd = torch.from_numpy(~greedy).to(dev)
            f = lambda a: torch.from_numpy(np.asarray(a)[vrow]).to(dev)  # noqa: E731
            P = processed_probs(x, f(b.temperature), f(b.top_k), f(b.top_p), f(b.min_p))
            Q = torch.zeros_like(P)
            # q of each draft position: the draft's distribution, or one-hot
            qrows = []
            for r_i, r in enumerate(sorted(set(vrow.tolist()))):
                sid = int(np.asarray(b.seq_ids)[np.asarray(b.sample_seq_row)[r]])
                qrows.append(drafted[sid][1])
            k_of = {}
            for m, r in enumerate(vrow.tolist()):
                k_of.setdefault(r, []).append(m)
            for (r, ms), qr in zip(sorted(k_of.items()), qrows):
                idx = torch.tensor(ms, device=dev)
                if qr is not None:
                    Q.index_copy_(0, idx, qr.float())
                else:
                    Q.index_put_((idx, d[idx]), torch.ones(len(ms), device=dev))
            pd = P.gather(1, d.view(-1, 1)).view(-1)
            qd = Q.gather(1, d.view(-1, 1)).view(-1).clamp_min(1e-20)
            u = torch.rand(pd.shape, generator=self.gen, device=dev)
            acc_r = u < (pd / qd)
            resid = (P - Q).clamp_min(0)
            s = resid.sum(1, keepdim=True)
            resid = torch.where(s > 0, resid / s.clamp_min(1e-30), P)
            draw = torch.multinomial(resid, 1, generator=self.gen).view(-1)
            acc = torch.where(rnd, acc_r, acc)
            alt = torch.where(rnd, draw, alt)
        lp_d = lsm.gather(1, d.view(-1, 1)).view(-1)
        lp_a = lsm.gather(1, alt.view(-1, 1)).view(-1)
        both = torch.stack([acc.float(), alt.float(), lp_d, lp_a]).cpu().numpy()
        return both[0] > 0.5, both[1].astype(np.int64), both[2], both[3]
