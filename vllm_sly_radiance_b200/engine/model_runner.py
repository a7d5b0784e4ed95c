"""Model runner: turns a scheduled batch into device tensors, runs the model, samples.

Per step the host packs all metadata (token ids, positions, query offsets, sequence lengths,
block tables, KV slot mapping, GDN state slots, attention row tiles) into one pinned buffer and
issues one host->device copy into persistent device buffers; every kernel reads views of those
buffers, so a decode batch can be replayed from a CUDA graph captured per batch-size bucket
(reference: vLLM V2 runner FULL decode graphs, capture sizes 8..64, ``README.md:261-262``).
Sampled token ids come back with one device->host copy.
"""
from __future__ import annotations

import math
import time
from dataclasses import dataclass
from typing import Optional

import numpy as np
import torch

from ..models.hybrid import HybridModel, ModelCaches, StepMeta
from .request import Request
from .sampler import SamplingTensors, apply_penalties, needs_full_vocab, row_seed, sample
from .scheduler import SchedulerOutput

GRAPH_BUCKETS = [1, 2, 4, 8, 16, 32, 48, 64, 96, 128]


@dataclass
class StepResult:
    sampled: dict                 # request_id -> list[int]
    logits: Optional[torch.Tensor] = None
    num_tokens: int = 0
    used_graph: bool = False


class _Layout:
    """Offsets of the packed int32 metadata buffer."""

    def __init__(self, max_tokens, max_seqs, max_blocks, max_tiles):
        self.max_tokens, self.max_seqs, self.max_blocks, self.max_tiles = \
            max_tokens, max_seqs, max_blocks, max_tiles
        o = 0
        self.ids = o; o += max_tokens
        self.pos = o; o += max_tokens
        self.tseq = o; o += max_tokens
        self.qsl = o; o += max_seqs + 1
        self.slen = o; o += max_seqs
        self.init = o; o += max_seqs
        self.slot = o; o += max_seqs
        self.tile_s = o; o += max_tiles
        self.tile_r = o; o += max_tiles
        self.commit = o; o += max_seqs
        self.bt = o; o += max_seqs * max_blocks
        self.size = o


class ModelRunner:
    def __init__(self, model: HybridModel, caches: ModelCaches, *, max_num_seqs: int,
                 max_num_tokens: int, max_model_len: int, device, enable_graphs: bool = True,
                 graph_max_bs: int = 64, num_spec_tokens: int = 0):
        self.model = model
        self.caches = caches
        self.device = torch.device(device)
        self.bs = caches.block_size
        self.max_seqs = max_num_seqs
        self.max_tokens = max(max_num_tokens, max_num_seqs * (1 + num_spec_tokens))
        self.max_blocks = (max_model_len + self.bs - 1) // self.bs + 1
        cfg = model.cfg
        attn_layers = [l for l in model.layers if l.is_attn]
        self.G = (attn_layers[0].mixer.Hq // attn_layers[0].mixer.Hkv) if attn_layers else 1
        self.Hkv = attn_layers[0].mixer.Hkv if attn_layers else 1
        self.max_tiles = (self.max_tokens * self.G + 63) // 64 + self.max_seqs
        self.L = _Layout(self.max_tokens, self.max_seqs, self.max_blocks, self.max_tiles)
        pin = self.device.type == "cuda"
        self.h_meta = torch.zeros(self.L.size, dtype=torch.int32, pin_memory=pin)
        self.h_slots = torch.zeros(self.max_tokens, dtype=torch.int64, pin_memory=pin)
        self.d_meta = torch.zeros(self.L.size, dtype=torch.int32, device=self.device)
        self.d_slots = torch.full((self.max_tokens,), -1, dtype=torch.int64, device=self.device)
        self.h_out = torch.zeros(self.max_tokens, dtype=torch.int64, pin_memory=pin)
        # the device status word's error code rides back with the sampled ids (same sync)
        self.h_status = torch.zeros(1, dtype=torch.int32, pin_memory=pin)
        self._status_staged = False
        self.step_count = 0
        self.num_spec_tokens = num_spec_tokens
        self.enable_graphs = enable_graphs and self.device.type == "cuda"
        self.graph_max_bs = min(graph_max_bs, max_num_seqs)
        self.graphs: dict = {}
        self.graph_pool = None
        self.last_timing = {}
        self._scratch: dict = {}
        self._h2d_event = None
        self.last_io = (0, 0)      # (host->device, device->host) bytes copied by the last step

    # ------------------------------------------------------------------------------------------
    # metadata
    # ------------------------------------------------------------------------------------------
    def _views(self, B: int, T: int, ntiles: int, nb: int) -> StepMeta:
        L, d = self.L, self.d_meta
        return StepMeta(
            num_seqs=B, num_tokens=T,
            query_start_loc=d[L.qsl:L.qsl + B + 1],
            seq_lens=d[L.slen:L.slen + B],
            has_initial=d[L.init:L.init + B],
            state_slots=d[L.slot:L.slot + B],
            block_tables=d[L.bt:L.bt + B * nb].view(B, nb),
            slot_mapping=self.d_slots[:T],
            positions=d[L.pos:L.pos + T],
            token_seq=d[L.tseq:L.tseq + T],
            tile_seq=d[L.tile_s:L.tile_s + ntiles],
            tile_row0=d[L.tile_r:L.tile_r + ntiles],
            _scratch=self._scratch)

    def _num_splits(self, B: int, ntiles: int, max_kv: int, decode: bool = False) -> int:
        """KV splits per (row tile, kv head): fill ~2 CTAs per SM, at least 256 keys per split
        (one 64-key tile for decode batches, whose per-tile work is small), at most 32.  The
        decode kernel merges up to 128 in-kernel, but more than 32 measured no faster at 16k
        context (41 us at 32 or 64 splits, 58 us at 128) and slower at 1.5k.  Sized for 128k keys
        or more (long-context engines), a decode split streams its keys one tile at a time for
        long enough that the loads in flight, not the merge, bound it: there the splits fill ~3
        CTAs per SM, up to 128."""
        ctas = max(1, ntiles * self.Hkv)
        if decode and max_kv >= 131072:
            return max(1, min(128, 148 * 3 // ctas, (max_kv + 1023) // 1024))
        s = max(1, min(32, 148 * 2 // ctas))
        s = min(s, max(1, (max_kv + (63 if decode else 255)) // (64 if decode else 256)))
        return s

    def prepare(self, out: SchedulerOutput, pad_to: Optional[int] = None, nb_fixed: Optional[int] = None):
        """Pack host metadata for the scheduled seqs.  With pad_to, the batch is padded to a graph
        bucket of pure decode rows (1 token each).  Returns (meta, input_ids view, sample index,
        per-seq sample counts)."""
        L = self.L
        # the pinned staging buffers are reused: the previous asynchronous upload must have
        # finished reading them before they are overwritten
        if self._h2d_event is not None:
            self._h2d_event.synchronize()
        h = self.h_meta.numpy()
        hs = self.h_slots.numpy()
        seqs = out.seqs
        B_real = len(seqs)
        B = pad_to or B_real
        bs = self.bs
        G = self.G
        qsl = [0]
        max_kv = 1
        nb = 1
        tok_ptr = 0
        tiles_s, tiles_r = [], []
        sample_idx = []
        sample_cnt = []
        for b in range(B):
            if b < B_real:
                s = seqs[b]
                req = s.req
                c0 = req.num_computed_tokens
                if s.is_decode:
                    toks = [req.all_token_ids[-1]] + list(s.draft_tokens)
                else:
                    toks = req.all_token_ids[c0:c0 + s.num_new_tokens]
                n = len(toks)
                h[L.ids + tok_ptr:L.ids + tok_ptr + n] = toks
                h[L.pos + tok_ptr:L.pos + tok_ptr + n] = np.arange(c0, c0 + n)
                h[L.tseq + tok_ptr:L.tseq + tok_ptr + n] = b
                blocks = req.block_ids
                pos = np.arange(c0, c0 + n)
                bidx = np.asarray(blocks, dtype=np.int64)[pos // bs]
                hs[tok_ptr:tok_ptr + n] = bidx * bs + pos % bs
                h[L.slen + b] = c0 + n
                h[L.init + b] = 1 if c0 > 0 else 0
                h[L.slot + b] = req.state_slot
                nbk = len(blocks)
                max_kv = max(max_kv, c0 + n)
                row = L.bt + b * (nb_fixed or self.max_blocks)
                if nb_fixed is None:
                    h[row:row + nbk] = blocks
                else:
                    h[row:row + min(nbk, nb_fixed)] = blocks[:nb_fixed]
                nb = max(nb, nbk)
                if s.samples:
                    if s.is_decode and s.draft_tokens:
                        sample_idx.extend(range(tok_ptr, tok_ptr + n))
                        sample_cnt.append(n)
                    else:
                        sample_idx.append(tok_ptr + n - 1)
                        sample_cnt.append(1)
                else:
                    sample_cnt.append(0)
            else:   # padded decode row -> dummy slot / block 0
                n = 1
                h[L.ids + tok_ptr] = 0
                h[L.pos + tok_ptr] = 0
                h[L.tseq + tok_ptr] = b
                hs[tok_ptr] = -1
                h[L.slen + b] = 1
                h[L.init + b] = 0
                h[L.slot + b] = 0
                row = L.bt + b * (nb_fixed or self.max_blocks)
                h[row] = 0
                sample_idx.append(tok_ptr)
            R = n * G
            for r0 in range(0, R, 64):
                tiles_s.append(b)
                tiles_r.append(r0)
            tok_ptr += n
            qsl.append(tok_ptr)
        T = tok_ptr
        h[L.qsl:L.qsl + B + 1] = qsl
        ntiles = len(tiles_s)
        h[L.tile_s:L.tile_s + ntiles] = tiles_s
        h[L.tile_r:L.tile_r + ntiles] = tiles_r
        if nb_fixed is not None:
            nb = nb_fixed
        else:
            # compact block table rows to width nb
            src = h[L.bt:L.bt + B * self.max_blocks].reshape(B, self.max_blocks)[:, :nb].copy()
            h[L.bt:L.bt + B * nb] = src.reshape(-1)
        # H2D
        end = L.bt + B * nb
        self._h2d_bytes = end * 4 + T * 8
        if self.device.type == "cuda":
            self.d_meta[:end].copy_(self.h_meta[:end], non_blocking=True)
            self.d_slots[:T].copy_(self.h_slots[:T], non_blocking=True)
            self._h2d_event = torch.cuda.Event()
            self._h2d_event.record()
        else:
            self.d_meta[:end].copy_(self.h_meta[:end])
            self.d_slots[:T].copy_(self.h_slots[:T])
        meta = self._views(B, T, ntiles, nb)
        # decode batches size the split count for the longest context, in graphs (replays keep
        # the captured count) and eagerly alike, so both paths compute identical numerics
        all_decode = all(s.is_decode for s in seqs)
        decode_rows = (pad_to or all_decode) and T == B and self.G <= 16
        meta.num_splits = self._num_splits(B, ntiles, self.max_blocks * bs if (pad_to or all_decode)
                                           else max_kv, decode=bool(decode_rows))
        ids = self.d_meta[L.ids:L.ids + T]
        return meta, ids, sample_idx, sample_cnt

    # ------------------------------------------------------------------------------------------
    # execution
    # ------------------------------------------------------------------------------------------
    def _forward_logits(self, ids, meta, sample_idx_t):
        hidden = self.model.forward(ids, meta, self.caches)
        return self.model.logits(hidden[sample_idx_t])

    def _graph_bucket(self, out: SchedulerOutput) -> Optional[int]:
        if not self.enable_graphs or not out.seqs:
            return None
        if any((not s.is_decode) or s.draft_tokens for s in out.seqs):
            return None
        B = len(out.seqs)
        for bk in GRAPH_BUCKETS:
            if bk >= B and bk <= self.graph_max_bs:
                return bk
        return None

    def execute(self, out: SchedulerOutput, want_logits: bool = False) -> StepResult:
        self.step_count += 1
        reqs = [s.req for s in out.seqs]
        bucket = self._graph_bucket(out)
        st = None
        if bucket is not None and not want_logits and not _needs_penalties(reqs):
            toks = self._run_graph(out, bucket)
            self.last_io = (self._h2d_bytes, 8 * bucket)
            sampled = {}
            for b, s in enumerate(out.seqs):
                sampled[s.req.request_id] = [int(toks[b])]
            return StepResult(sampled, num_tokens=len(out.seqs), used_graph=True)
        meta, ids, sample_idx, sample_cnt = self.prepare(out)
        sample_idx_t = torch.tensor(sample_idx, dtype=torch.long).to(self.device, non_blocking=True)
        logits = self._forward_logits(ids, meta, sample_idx_t)
        sreqs = []
        for s, c in zip(out.seqs, sample_cnt):
            sreqs.extend([s.req] * c)
        sampled = {}
        h2d = self._h2d_bytes + 8 * len(sample_idx)
        d2h = 0
        if sreqs:
            h2d += len(sreqs) * (4 + 4 + 4 + 4 + 8)
            d2h = 8 * len(sreqs)
            st = SamplingTensors.from_requests(sreqs, self.device)
            lg = apply_penalties(logits, sreqs)
            toks, _, _ = sample(lg, st, 0)
            self.h_out[:len(sreqs)].copy_(toks, non_blocking=True) if self.device.type == "cuda" \
                else self.h_out[:len(sreqs)].copy_(toks)
            if self.device.type == "cuda":
                self._stage_status()
                torch.cuda.current_stream().synchronize()
            hv = self.h_out[:len(sreqs)].tolist()
            j = 0
            for s, c in zip(out.seqs, sample_cnt):
                if c:
                    sampled[s.req.request_id] = hv[j:j + c] if c == 1 else hv[j:j + c]
                    j += c
        self.last_io = (h2d, d2h)
        return StepResult(sampled, logits=logits if want_logits else None,
                          num_tokens=meta.num_tokens)

    def _stage_status(self):
        """Queue the copy of the device error code next to the step's output copy."""
        from ..ops import kernels as K
        self.h_status.copy_(K.status_word(self.device)[:1], non_blocking=True)
        self._status_staged = True

    def read_status(self) -> int:
        """Error code the step's kernels recorded (0 = ok).  Free when the step already synced
        its output copy; otherwise one 4-byte copy and a stream sync."""
        if self.device.type != "cuda":
            return 0
        if not self._status_staged:
            self._stage_status()
            torch.cuda.current_stream().synchronize()
        self._status_staged = False
        return int(self.h_status[0])

    # ------------------------------------------------------------------------------------------
    # CUDA graphs (pure decode batches)
    # ------------------------------------------------------------------------------------------
    def _graph_inputs(self, bucket):
        g = self.graphs.get(bucket)
        return g

    def _run_graph(self, out: SchedulerOutput, bucket: int):
        nb_fixed = self.max_blocks
        meta, ids, sample_idx, _ = self.prepare(out, pad_to=bucket, nb_fixed=nb_fixed)
        reqs = [s.req for s in out.seqs]
        greedy = all(r.params.greedy for r in reqs)
        mode = "greedy" if greedy else ("full" if needs_full_vocab(reqs) else "window")
        key = (bucket, mode)
        g = self.graphs.get(key)
        if g is None:
            # warm up and capture on an all-padding batch (dummy state slot / KV block 0), so the
            # capture never advances the real sequences' GDN state; then restore the real batch
            from .scheduler import SchedulerOutput as _SO
            dmeta, dids, _, _ = self.prepare(_SO([], 0, [], []), pad_to=bucket, nb_fixed=nb_fixed)
            g = self._capture(bucket, mode, dmeta, dids)
            self.graphs[key] = g
            meta, ids, sample_idx, _ = self.prepare(out, pad_to=bucket, nb_fixed=nb_fixed)
        # sampling params into the static buffers
        B = len(reqs)
        if not greedy:
            self._h2d_bytes += B * (4 + 4 + 4 + 4 + 8)
            g["temp"][:B].copy_(torch.tensor([r.params.temperature for r in reqs]), non_blocking=True)
            g["topk"][:B].copy_(torch.tensor([r.params.top_k for r in reqs], dtype=torch.int32), non_blocking=True)
            g["topp"][:B].copy_(torch.tensor([r.params.top_p for r in reqs]), non_blocking=True)
            g["minp"][:B].copy_(torch.tensor([r.params.min_p for r in reqs]), non_blocking=True)
            # the captured sampler reads a per-row Philox seed; fold the step in on the host
            g["seed"][:B].copy_(torch.tensor([row_seed(r) for r in reqs], dtype=torch.int64),
                                non_blocking=True)
        g["graph"].replay()
        self.h_out[:bucket].copy_(g["out"], non_blocking=True)
        self._stage_status()
        torch.cuda.current_stream().synchronize()
        return self.h_out[:B].tolist()

    def capture_all(self):
        """Capture the decode graphs of every bucket (greedy and sampled) up front, on dummy
        all-padding batches, so no request pays a capture inside its step."""
        if not self.enable_graphs:
            return
        from .scheduler import SchedulerOutput as _SO
        for bucket in GRAPH_BUCKETS:
            if bucket > self.graph_max_bs:
                break
            # the full-vocabulary mode (top_k disabled) is captured when a batch first needs it
            for mode in ("greedy", "window"):
                if (bucket, mode) in self.graphs:
                    continue
                dmeta, dids, _, _ = self.prepare(_SO([], 0, [], []), pad_to=bucket,
                                                 nb_fixed=self.max_blocks)
                self.graphs[(bucket, mode)] = self._capture(bucket, mode, dmeta, dids)
        torch.cuda.synchronize(self.device)

    def _capture(self, bucket, mode, meta, ids):
        """mode: 'greedy' (argmax), 'window' (top-64 window draw, every top_k in 1..64) or
        'full' (full-vocabulary draw).  Sampled graphs always apply min_p (0 = off)."""
        dev = self.device
        greedy = mode == "greedy"
        sidx = torch.arange(bucket, dtype=torch.long, device=dev)
        temp = torch.zeros(bucket, dtype=torch.float32, device=dev)
        topk = torch.full((bucket,), 1 if mode == "window" else 0, dtype=torch.int32, device=dev)
        topp = torch.ones(bucket, dtype=torch.float32, device=dev)
        minp = torch.zeros(bucket, dtype=torch.float32, device=dev)
        seed = torch.zeros(bucket, dtype=torch.int64, device=dev)
        step = torch.zeros(1, dtype=torch.int64, device=dev)
        st = SamplingTensors(temp, topk, topp, minp, seed, greedy, True, mode == "full")

        def run():
            lg = self._forward_logits(ids, meta, sidx)
            if greedy:
                from ..ops import kernels as K
                return K.argmax(lg)
            toks, _, _ = sample(lg, st, 0)
            return toks

        # warm up outside the graph (allocator, TMA maps, attribute setup)
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            for _ in range(2):
                run()
        torch.cuda.current_stream().wait_stream(s)
        graph = torch.cuda.CUDAGraph()
        if self.graph_pool is None:
            self.graph_pool = torch.cuda.graph_pool_handle()
        with torch.cuda.graph(graph, pool=self.graph_pool):
            out = run()
        # every tensor the graph reads must outlive it: a freed input's memory is handed to the
        # next eager allocation and the replay would read whatever that step wrote there
        return dict(graph=graph, out=out, temp=temp, topk=topk, topp=topp, seed=seed, step=step,
                    sidx=sidx, minp=minp, st=st)


def _needs_penalties(reqs) -> bool:
    return any(r.params.presence_penalty or r.params.frequency_penalty or
               r.params.repetition_penalty != 1.0 for r in reqs)
