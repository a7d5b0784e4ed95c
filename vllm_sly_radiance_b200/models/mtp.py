"""Multi-token-prediction (MTP) drafter: the target's own next-next-token head as the proposer.

Reference behaviour: the Qwen3-Next MTP head served as the drafter (k = 4) in the reference's
alternative speculative path (``serve-mxfp4.sh:455-465``, ``radiance_draft.py``,
``patch_mtp_*``).  One MTP module: the embedding of token t_{p+1} and the target's hidden state
h_p are each RMS-normed, concatenated and projected back to the hidden size (fc, 2H -> H); one
full-attention decoder layer of the target's geometry (its own paged K/V, indexed by the target's
block tables) and the shared final norm + lm_head then predict t_{p+2}.  Drafting chains the
module: its output hidden state and the drafted token feed the next step.

Bookkeeping: MTP cache position p holds the layer's K/V for the pair (h_p, t_{p+1}).  After each
target step ``observe`` runs the module over every committed row (prefill chunks, the accepted
prefix of a verified block) paired with its next token, which rewrites the speculative entries of
the previous proposal; the output at a request's last committed row is already the first draft.
``propose`` runs the remaining k - 1 single-row steps.
"""
from __future__ import annotations

import torch

from ..ops import kernels as K
from .hybrid import AttentionMixer, MLP, StepMeta, TPInfo, rope_cache
from .layers import Linear
from .weights import RandomWeights


class MTPDrafter:
    aux_layers = None          # conditions on the target's final hidden states only

    def __init__(self, target, k: int, device, block_size: int, num_blocks: int, seed: int = 3,
                 window: int = 16):
        cfg = target.cfg
        self.cfg = cfg
        self.target = target
        self.k = k
        self.window = window
        self.device = torch.device(device)
        quant = target.quant
        W = RandomWeights(cfg, seed, self.device)
        H = cfg.hidden_size
        self.enorm = W.tensor("mtp.enorm", (H,), "norm")
        self.hnorm = W.tensor("mtp.hnorm", (H,), "norm")
        self.fc = Linear(W.linear("mtp.fc", H, 2 * H), quant, "mtp_fc")
        self.ln1 = W.tensor("mtp.ln1", (H,), "norm")
        self.ln2 = W.tensor("mtp.ln2", (H,), "norm")
        tp = TPInfo()
        self.attn = AttentionMixer(cfg, tp, quant, W, "mtp.")
        self.mlp = MLP(cfg, tp, quant, W, "mtp.")
        self.final_norm = W.tensor("mtp.final_norm", (H,), "norm")
        if self.device.type == "cuda":
            self.attn.cos_sin = rope_cache(cfg.max_position_embeddings, cfg.rotary_dim,
                                           cfg.rope_theta, self.device)
        kv_dt = torch.float8_e4m3fn if quant in ("mxfp4", "fp8") else torch.bfloat16
        self.kc = torch.zeros(num_blocks, self.attn.Hkv, block_size, cfg.head_dim, dtype=kv_dt,
                              device=self.device)
        self.vc = torch.zeros_like(self.kc)
        self.bs = block_size
        self.kv = None                     # engine KV manager (block allocation)
        self.pending = {}                  # request id -> (first draft, hidden, position, T)
        self.last = {}                     # request id -> (window ids [k, W], probs [k, W])

    @staticmethod
    def for_engine(engine, k: int) -> "MTPDrafter":
        d = MTPDrafter(engine.model, k, engine.device, engine.config.block_size, engine.num_blocks)
        d.kv = engine.kv
        return d

    # ------------------------------------------------------------------------------------------
    def _meta(self, reqs_rows: list) -> StepMeta:
        """reqs_rows: [(request, [positions])] -> metadata for rows at those MTP positions (each
        attends to its request's MTP entries up to its own position)."""
        dev = self.device
        bs = self.bs
        G = self.attn.Hq // self.attn.Hkv
        qsl, lens, slots, pos, tseq, tiles_s, tiles_r, bts = [0], [], [], [], [], [], [], []
        maxb = 1
        for b, (r, ps) in enumerate(reqs_rows):
            need = (ps[-1] + 1 + bs - 1) // bs
            if self.kv is not None and len(r.block_ids) < need:
                self.kv.allocate(r, ps[-1] + 1)
            blocks = list(r.block_ids)
            while len(blocks) < need:
                blocks.append(0)              # pool exhausted: unwritten dummy page
            bts.append(blocks)
            maxb = max(maxb, len(blocks))
            for p in ps:
                ok = p // bs < len(r.block_ids)
                slots.append(blocks[p // bs] * bs + p % bs if ok else -1)
                pos.append(p)
                tseq.append(b)
            qsl.append(qsl[-1] + len(ps))
            lens.append(ps[-1] + 1)
            for r0 in range(0, len(ps) * G, 64):
                tiles_s.append(b)
                tiles_r.append(r0)
        bt = torch.zeros(len(reqs_rows), maxb, dtype=torch.int32)
        for i, b in enumerate(bts):
            bt[i, :len(b)] = torch.tensor(b, dtype=torch.int32)
        i32 = lambda v: torch.tensor(v, dtype=torch.int32, device=dev)
        return StepMeta(num_seqs=len(reqs_rows), num_tokens=len(pos),
                        query_start_loc=i32(qsl), seq_lens=i32(lens),
                        has_initial=i32([1] * len(reqs_rows)),
                        state_slots=i32([0] * len(reqs_rows)), block_tables=bt.to(dev),
                        slot_mapping=torch.tensor(slots, dtype=torch.int64, device=dev),
                        positions=i32(pos), token_seq=i32(tseq), tile_seq=i32(tiles_s),
                        tile_row0=i32(tiles_r), num_splits=1)

    def _module(self, h, toks, meta):
        """One MTP pass over rows (h_p, t_{p+1}) -> (output hidden [n, H], logits [n, V])."""
        eps = self.cfg.rms_norm_eps
        e = self.target.embed[toks]
        en, _ = K.add_rms_norm(e, None, self.enorm, eps, want_residual=False)
        hn, _ = K.add_rms_norm(h.to(torch.bfloat16), None, self.hnorm, eps, want_residual=False)
        x = self.fc(torch.cat([en, hn], 1).contiguous())
        n, res = K.add_rms_norm(x, None, self.ln1, eps)
        a = self.attn.forward(n, meta, self.kc, self.vc)
        n, res = K.add_rms_norm(a, res, self.ln2, eps)
        m = self.mlp.forward(n)
        out = (res.float() + m.float()).to(torch.bfloat16)
        fn, _ = K.add_rms_norm(out, None, self.final_norm, eps, want_residual=False)
        return out, self.target.logits(fn).float()

    def _choose(self, logits, reqs):
        """Draft token + its window (top-W ids, probabilities) per row: argmax at T = 0, a draw
        from the renormalised top-W window otherwise."""
        W = min(self.window, logits.shape[-1])
        vals, ids = torch.topk(logits, W, dim=-1)
        temps = torch.tensor([max(r.params.temperature, 0.0) for r in reqs],
                             device=logits.device).view(-1, 1)
        greedy = temps <= 0
        p = torch.softmax(vals / temps.clamp(min=1e-6), -1)
        onehot = torch.zeros_like(p)
        onehot[:, 0] = 1.0
        p = torch.where(greedy, onehot, p)
        pick = torch.where(greedy.view(-1), torch.zeros_like(ids[:, 0]),
                           torch.multinomial(p, 1).view(-1))
        tok = ids.gather(1, pick.view(-1, 1)).view(-1)
        return tok, ids, p

    # ------------------------------------------------------------------------------------------
    def observe(self, sched, meta, aux, sampled: dict, sample_cnt, hidden=None):
        """Rewrite the MTP entries of every row the target committed this step and keep the
        first draft of every request that sampled."""
        if hidden is None:
            return
        qsl = meta.query_start_loc.cpu().tolist()
        pos_all = meta.positions.cpu().tolist()
        rows, toks, groups = [], [], []
        for bi, s in enumerate(sched.seqs):
            r = s.req
            new = sampled.get(r.request_id)
            r0 = qsl[bi]
            ps, tk = [], []
            if s.is_decode:
                # plain decode: one row; verify: the accepted prefix (1 + accepted rows), each
                # paired with the token committed after it
                for j, nt in enumerate(new or []):
                    ps.append(pos_all[r0 + j])
                    tk.append(nt)
            else:
                for j in range(s.num_new_tokens):
                    p = pos_all[r0 + j]
                    if p + 1 < r.num_prompt_tokens:
                        nt = r.prompt_token_ids[p + 1]
                    elif new:
                        nt = new[0]                 # the prompt's last row: the sampled token
                    else:
                        break
                    ps.append(p)
                    tk.append(nt)
            if ps:
                rows.extend(range(r0, r0 + len(ps)))
                groups.append((r, ps, bool(new)))
                toks.extend(tk)
        if not rows:
            return
        dev = self.device
        h = hidden[torch.tensor(rows, dtype=torch.long, device=dev)]
        mm = self._meta([(r, ps) for r, ps, _ in groups])
        out, logits = self._module(h, torch.tensor(toks, dtype=torch.long, device=dev), mm)
        last_rows, last_reqs = [], []
        o = 0
        for r, ps, has_new in groups:
            o += len(ps)
            if has_new:
                last_rows.append(o - 1)
                last_reqs.append((r, ps[-1]))
        if not last_rows:
            return
        lr = torch.tensor(last_rows, dtype=torch.long, device=dev)
        tok, ids, p = self._choose(logits[lr], [r for r, _ in last_reqs])
        for i, (r, pos) in enumerate(last_reqs):
            self.pending[r.request_id] = (tok[i:i + 1], out[lr[i]:lr[i] + 1], pos,
                                          ids[i:i + 1], p[i:i + 1])

    def propose(self, reqs, new_tokens) -> list[list[int]]:
        live = [r for r in reqs if r.request_id in self.pending]
        if not live:
            return [[] for _ in reqs]
        dev = self.device
        tok = torch.cat([self.pending[r.request_id][0] for r in live])
        h = torch.cat([self.pending[r.request_id][1] for r in live])
        pos = [self.pending[r.request_id][2] for r in live]
        win_ids = [[self.pending[r.request_id][3]] for r in live]
        win_p = [[self.pending[r.request_id][4]] for r in live]
        drafts = [tok]
        for j in range(1, self.k):
            mm = self._meta([(r, [p + j]) for r, p in zip(live, pos)])
            h, logits = self._module(h, tok, mm)
            tok, ids, p = self._choose(logits, live)
            drafts.append(tok)
            for i in range(len(live)):
                win_ids[i].append(ids[i:i + 1])
                win_p[i].append(p[i:i + 1])
        D = torch.stack(drafts, 1).cpu().tolist()
        by_id = {}
        for i, r in enumerate(live):
            by_id[r.request_id] = D[i]
            self.last[r.request_id] = (torch.cat(win_ids[i]), torch.cat(win_p[i]))
            del self.pending[r.request_id]
        return [by_id.get(r.request_id, []) for r in reqs]

    def draft_windows(self, reqs, k, dev):
        ids = torch.stack([self.last[r.request_id][0][:k] for r in reqs])
        pr = torch.stack([self.last[r.request_id][1][:k] for r in reqs])
        return ids.to(dev), pr.to(dev)
