"""The System One API (src/d1.ts) over the B200 engines.

Decision.load / systemOne / systemOneBatch / probabilities / probabilitiesBatch / destroy keep the reference's
names, argument meaning and error behaviour. Differences, all on purpose:
  - `devices` (a list of CUDA device indices) spreads whole requests over GPUs: each device holds a full weight
    replica and runs its own passes; results come back in request order. WebGPU-only options (matrixUnits,
    device, fetch, directWeights) are accepted and ignored.
  - The encoder (EmbeddingGemma-architecture) also exposes `embed(seqs)`: Eg2Engine.embed's mean-pooled,
    L2-normalised embeddings. Its typed-decision head (src/eg2-head.ts), which the reference runs on the host, runs
    on the GPU here (dc_eg2_head), one launch per batch.
  - With the model's tokenizer.json and tokenizer_config.json beside the weights (as the reference's exports ship
    them), states and questions are the reference's: any JSON state and {type, instructions, criteria} questions,
    rendered and tokenized by decision_js_b200.prompts. Without them, requests arrive tokenized: a decoder
    request's state is its trunk token ids and each question carries `branch` (its token ids) and `groups` (per
    option, the token ids whose best logit scores it), exactly what D13BPrompt produces (src/d1-3b-prompt.ts)
    and D13BEngine.run consumes (src/d1-3b-engine.ts:12-14); an EmbeddingGemma 2 request's state is the token
    ids of its text and each question carries `question_ids` and `option_ids` (one list per option), each as
    the model embeds it (<bos> prompt + text <eos>, src/eg2-prompt.ts:43-46).
"""
from __future__ import annotations

import concurrent.futures as cf
import ctypes
import itertools
import json
import os
import threading

import numpy as np

from collections import OrderedDict

from . import _lib, prompts
from ._lib import Context, DecisionError, check, lib
from .questions import answer, check_question, softmax


def passes(sizes, budget):
    """Whole requests per pass up to `budget` tokens (src/d1.ts:130-133): a pass always takes at least one
    request, then adds requests while they fit. Returns [(i, j)] index ranges."""
    out, i = [], 0
    while i < len(sizes):
        j, used = i, 0
        while True:
            used += sizes[j]
            j += 1
            if not (j < len(sizes) and used + sizes[j] <= budget):
                break
        out.append((i, j))
        i = j
    return out


def shard(sizes, n):
    """Contiguous, token-balanced shards of a request list over n workers: [(i, j)] per worker (possibly
    empty). Shard boundaries fall where the running token count crosses k/n of the total."""
    total = float(sum(sizes))
    bounds, acc, k = [0], 0.0, 1
    for idx, s in enumerate(sizes):
        acc += s
        while k < n and acc >= total * k / n:
            bounds.append(idx + 1)
            k += 1
    while len(bounds) < n:
        bounds.append(len(sizes))
    bounds.append(len(sizes))
    return [(bounds[w], bounds[w + 1]) for w in range(n)]


class _Model:
    """One device's context and weight replica."""

    def __init__(self, base: str, device: int):
        self.h = None
        self.ctx = Context(device)
        h = ctypes.c_void_p()
        try:
            check(lib().dc_load_weights(self.ctx.h, base.encode(), ctypes.byref(h)))
        except BaseException:
            self.ctx.close()
            raise
        self.h = h
        buf = ctypes.create_string_buffer(64)
        check(lib().dc_model_kind(h, buf, 64))
        self.kind = buf.value.decode()
        e = self.cfg("embed_dim")  # read once here: embed() must not touch a handle another thread may free
        self.embed_dim = int(e) if e else None

    def cfg(self, key: str, default=None):
        v = ctypes.c_double()
        if lib().dc_model_config_f(self.h, key.encode(), ctypes.byref(v)) != 0:
            return default
        return v.value

    def close(self):
        """Frees the weights, then the context (a model's buffers are freed on its context's device and stream)."""
        if getattr(self, "ctx", None) is not None and self.ctx.h:
            self.free_buffers()
        if getattr(self, "h", None):
            lib().dc_model_free(self.h)
            self.h = None
        ctx = getattr(self, "ctx", None)  # absent when dc_init itself failed
        if ctx is not None:
            ctx.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    # ---------------------------------------------------------------- one pass
    def encoder_pass(self, seqs):
        ids = np.concatenate([np.asarray(s, np.int32) for s in seqs])
        lens = np.array([len(s) for s in seqs], np.int64)
        ends = np.cumsum(lens)
        bounds = np.stack([ends - lens, ends], 1).astype(np.int32)
        N = self._out_rows()
        out = np.empty((len(seqs), N), np.float32)
        check(lib().dc_forward_encoder(self.h, ids.ctypes.data, bounds.ctypes.data, int(ids.size), len(seqs),
                                       out.ctypes.data))
        return out

    def _out_rows(self):
        """Width of the pooled output: the projection's rows, else the hidden size (looked up once)."""
        if getattr(self, "_n_out", None) is None:
            try:
                self._n_out = self._proj_rows()
            except DecisionError:
                self._n_out = int(self.cfg("hidden"))
        return self._n_out

    def _proj_rows(self):
        rows = ctypes.c_int64()
        check(lib().dc_model_tensor(self.h, b"projection", None, None, None, ctypes.byref(rows), None))
        return int(rows.value)

    def _dbuf(self, name, nbytes):
        """A grow-only device buffer of this replica's context (freed with the context)."""
        bufs = self.__dict__.setdefault("_bufs", {})
        have = bufs.get(name)
        if have is None or have[1] < nbytes:
            if have is not None:
                lib().dc_free(self.ctx.h, have[0])
            p = ctypes.c_void_p()
            check(lib().dc_alloc(self.ctx.h, max(nbytes, 256), ctypes.byref(p)))
            bufs[name] = (p, max(nbytes, 256))
        return bufs[name][0]

    def head_logits(self, S, Q, O, items):
        """EmbeddingGemma 2's decision head on the GPU (dc_eg2_head): the raw logit of every option of every
        question instance. S, Q, O [n, E] f32 normalised embeddings; items [n_items, 6] int32."""
        arrs = [np.ascontiguousarray(a) for a in (S.astype(np.float32), Q.astype(np.float32),
                                                     O.astype(np.float32), items.astype(np.int32))]
        n_out = int((items[:, 4] + items[:, 5]).max()) if len(items) else 0
        ptrs = []
        for name, a in zip(("hS", "hQ", "hO", "hI"), arrs):
            d = self._dbuf(name, a.nbytes)
            check(lib().dc_upload(self.ctx.h, d, a.ctypes.data, a.nbytes))
            ptrs.append(d)
        dout = self._dbuf("hL", 4 * max(n_out, 1))
        check(lib().dc_eg2_head(self.h, ptrs[0], len(S), ptrs[1], len(Q), ptrs[2], len(O), ptrs[3], len(items), dout))
        self.ctx.sync()
        out = np.empty(n_out, np.float32)
        check(lib().dc_download(self.ctx.h, out.ctypes.data, dout, out.nbytes))
        return out

    def free_buffers(self):
        for p, _ in self.__dict__.pop("_bufs", {}).values():
            lib().dc_free(self.ctx.h, p)

    def omni_pass(self, seqs):
        """D1OmniEngine.logits (dc_forward_omni): each sequence's raw logits at its option markers."""
        ids, pos, rng, taps, qtype, markers = omni_pack(seqs)
        out = np.empty(len(markers), np.float32)
        check(lib().dc_forward_omni(self.h, ids.ctypes.data, pos.ctypes.data, rng.ctypes.data, taps.ctypes.data,
                                    int(ids.size), qtype.ctypes.data, markers.ctypes.data, len(markers),
                                    out.ctypes.data))
        res, k = [], 0
        for s in seqs:
            res.append(out[k:k + len(s[1])])
            k += len(s[1])
        return res

    def laya_pass(self, seqs):
        """LayaEngine.logits (dc_forward_laya): each sequence's raw logits at its option markers."""
        ids, pos, rng, win, qtype, markers = laya_pack(seqs, int(self.cfg("window", 64)))
        out = np.empty(len(markers), np.float32)
        check(lib().dc_forward_laya(self.h, ids.ctypes.data, pos.ctypes.data, rng.ctypes.data, win.ctypes.data,
                                    int(ids.size), qtype.ctypes.data, markers.ctypes.data, len(markers),
                                    out.ctypes.data))
        res, k = [], 0
        for s in seqs:
            res.append(out[k:k + len(s[1])])
            k += len(s[1])
        return res

    def d3_pass(self, seqs, groups=None):
        """D3Engine.logits (dc_forward_d3): each sequence's raw code logits, options in order."""
        ids, pos, rng, spans, pairs = d3_pack(seqs, groups)
        out = np.empty(len(pairs), np.float32)
        check(lib().dc_forward_d3(self.h, ids.ctypes.data, pos.ctypes.data, rng.ctypes.data, int(ids.size),
                                  spans.ctypes.data, len(spans), pairs.ctypes.data, len(pairs), out.ctypes.data))
        res, k = [], 0
        for _, options in seqs:
            res.append(out[k:k + options])
            k += options
        return res

    def decoder_pass(self, trees):
        ids, pos, rng, leaves, leaf_ids = forest(trees)
        lens = np.fromiter((len(g) for g in leaf_ids), np.int64, count=len(leaf_ids))
        n = int(lens.max())
        flat = np.zeros((len(leaf_ids), n), np.int32)  # each readout's ids, padded with id 0
        flat[np.arange(n)[None, :] < lens[:, None]] = np.fromiter(itertools.chain.from_iterable(leaf_ids), np.int32,
                                                                  count=int(lens.sum()))
        out = np.empty((len(leaves), n), np.float32)
        check(lib().dc_forward_decoder(self.h, ids.ctypes.data, pos.ctypes.data, rng.ctypes.data, int(ids.size),
                                       leaves.ctypes.data, flat.ctypes.data, int(leaves.size), n, out.ctypes.data))
        return readout_scores(trees, out)


def forest(trees):
    """The packed forest of D13BEngine.run (src/d1-3b-engine.ts:46-68) as arrays: token ids, positions, key
    ranges [T, 4] (a trunk token reads [start, t+1); a branch token reads the trunk [start, start+p) and its own
    branch up to itself), readout rows (the last token of each branch) and each readout's ids (its groups,
    flattened). Built per segment (a trunk or a branch), then spread to tokens with np.repeat, all in int32."""
    seg_len, seg_trunk, p_seg, ts_idx, toks, leaf_ids = [], [], [], [], [], []
    for tr in trees:
        trunk = tr["trunk"]
        p = len(trunk)
        ti = len(seg_len)  # this tree's trunk segment
        toks.append(trunk)
        seg_len.append(p)
        seg_trunk.append(True)
        p_seg.append(p)
        ts_idx.append(ti)
        for b, br in enumerate(tr["branches"]):
            toks.append(br)
            seg_len.append(len(br))
            seg_trunk.append(False)
            p_seg.append(p)
            ts_idx.append(ti)
            leaf_ids.append([i for g in tr["groups"][b] for i in g])
    seg_len = np.asarray(seg_len, np.int32)
    seg_trunk = np.asarray(seg_trunk, bool)
    seg_start = np.zeros_like(seg_len)
    np.cumsum(seg_len[:-1], out=seg_start[1:])
    T = int(seg_start[-1] + seg_len[-1]) if seg_len.size else 0
    ids = np.fromiter(itertools.chain.from_iterable(toks), np.int32, count=T)
    ts = seg_start[np.asarray(ts_idx, np.int64)]  # per segment: its tree's start
    p = np.asarray(p_seg, np.int32)  # per segment: its tree's trunk length
    A = np.arange(T, dtype=np.int32)
    trunk_tok = np.repeat(seg_trunk, seg_len)
    pos = A - np.repeat(seg_start - np.where(seg_trunk, 0, p), seg_len)
    rng = np.empty((T, 4), np.int32)
    rng[:, 0] = np.repeat(ts, seg_len)
    rng[:, 1] = np.where(trunk_tok, A + 1, np.repeat(ts + p, seg_len))
    rng[:, 2] = np.repeat(np.where(seg_trunk, 0, seg_start), seg_len)
    rng[:, 3] = np.where(trunk_tok, 0, A + 1)
    br = ~seg_trunk
    leaves = seg_start[br] + seg_len[br] - 1
    return ids, pos, rng, leaves, leaf_ids


def d3_pack(seqs, groups=None):
    """The token axis of one d3-lite pass (src/d3-engine.ts:71-92): seqs are (ids, options); groups (sequences
    per request, consecutive) share their longest common token prefix as one trunk, read once, with at least one
    token left per sequence. Per token: id, position in its sequence, key ranges (its sequence, or the trunk and its
    own branch); per sequence the linear layers' two spans (a start, a length | write-a << 31, b start, b length;
    the first branch writes the trunk); per option a readout pair (the sequence's last token, code)."""
    ids, pos, rng, spans, pairs = [], [], [], [], []
    si = 0
    for n in (groups or [1] * len(seqs)):
        group = seqs[si:si + n]
        si += n
        P = 0
        if n > 1:
            first = group[0][0]
            lim = min(len(s[0]) for s in group) - 1
            while P < lim and all(s[0][P] == first[P] for s in group):
                P += 1
        ts = len(ids)
        ids.extend(group[0][0][:P])
        pos.extend(range(P))
        rng.extend([(ts, ts + P, 0, 0)] * P)
        for b, (sids, options) in enumerate(group):
            bs = len(ids)
            be = bs + len(sids) - P
            ids.extend(sids[P:])
            pos.extend(range(P, len(sids)))
            rng.extend([(ts, ts + P, bs, be) if P else (bs, be, 0, 0)] * (be - bs))
            flag = 0x80000000 if (b == 0 or not P) else 0
            spans.append((ts, P | flag, bs, be - bs) if P else (bs, (be - bs) | flag, 0, 0))
            pairs.extend((be - 1, k) for k in range(options))
    return (np.asarray(ids, np.int32), np.asarray(pos, np.int32), np.asarray(rng, np.int32).reshape(-1, 4),
            np.asarray(spans, np.uint32).reshape(-1, 4), np.asarray(pairs, np.int32).reshape(-1, 2))


OMNI_TYPES = {"choice": 0, "score": 1, "noul": 2}


def omni_pack(seqs):
    """The token axis of one d1-omni pass (src/omni-engine.ts:58-69): seqs are (ids, markers within the sequence,
    question type). Per token: id, position, key ranges (its whole sequence: bidirectional), the conv taps (t-1, t,
    t+1, never across sequences) and the question type; the markers as token rows."""
    lens = np.fromiter((len(s[0]) for s in seqs), np.int64, count=len(seqs))
    ends = np.cumsum(lens)
    starts = ends - lens
    T = int(ends[-1]) if len(seqs) else 0
    ids = np.fromiter(itertools.chain.from_iterable(s[0] for s in seqs), np.int32, count=T)
    seq_of = np.repeat(np.arange(len(seqs)), lens)
    t = np.arange(T, dtype=np.int64)
    st, en = starts[seq_of], ends[seq_of]
    pos = (t - st).astype(np.int32)
    rng = np.zeros((T, 4), np.int32)
    rng[:, 0], rng[:, 1] = st, en
    taps = np.zeros((T, 4), np.int32)
    taps[:, 0] = np.where(t > st, t - 1, -1)
    taps[:, 1] = t
    taps[:, 2] = np.where(t + 1 < en, t + 1, -1)
    qtype = np.repeat(np.fromiter((s[2] for s in seqs), np.int32, count=len(seqs)), lens).astype(np.int32)
    markers = np.fromiter((starts[i] + m for i, s in enumerate(seqs) for m in s[1]), np.int32)
    return ids, pos, rng, taps, qtype, markers


def laya_pack(seqs, window):
    """The token axis of one Laya pass (src/laya-engine.ts:52-63): omni_pack's ids, positions, whole-sequence key
    ranges, types and markers, and each token's window [max(start, t - window), min(end, t + window + 1)) for the
    local layers."""
    ids, pos, rng, _, qtype, markers = omni_pack(seqs)
    t = np.arange(ids.size)
    win = np.zeros_like(rng)
    win[:, 0] = np.maximum(rng[:, 0], t - window)
    win[:, 1] = np.minimum(rng[:, 1], t + window + 1)
    return ids, pos, rng, win, qtype, markers


def readout_scores(trees, out):
    """Option scores [tree][question][option] from the readout logits `out` [leaves, ids]: each option scores its
    best form, the max over its group's ids (src/d1-3b-engine.ts:111-121). Readouts that share a group layout are
    reduced together."""
    layouts, leaf = {}, 0
    for tr in trees:
        for groups in tr["groups"]:
            layouts.setdefault(tuple(len(g) for g in groups), []).append(leaf)
            leaf += 1
    flat = [None] * leaf
    for lens, rows in layouts.items():
        if min(lens, default=0) < 1:
            raise DecisionError(_lib.DC_EINVAL, "decision.js: an option has no token forms")
        offs = np.zeros(len(lens), np.int64)
        offs[1:] = np.cumsum(lens)[:-1]
        best = np.maximum.reduceat(out[rows][:, :int(sum(lens))], offs, axis=1)
        for r, vals in zip(rows, best.tolist()):
            flat[r] = vals
    scores, leaf = [], 0
    for tr in trees:
        scores.append(flat[leaf:leaf + len(tr["groups"])])
        leaf += len(tr["groups"])
    return scores


class Decision:
    """D1 / Decision (src/d1.ts:38-227) on one or more B200s."""

    def __init__(self, models, kind: str, tokens_per_pass: int, config: dict | None = None, tokenizer=None,
                 workflow: str = ""):
        self.models = models
        self.kind = kind
        self.tokens_per_pass = tokens_per_pass
        self.config = config or {}
        self.tokenizer = tokenizer
        self.workflow = workflow  # EmbeddingGemma 2: the workflow named in every state's text (src/d1.ts:26-28)
        self._prompt3b = None
        self.shareState = False  # d3-lite: one trunk per request for its questions (src/d1.ts:21-24, 51-52)
        self._emb = OrderedDict()  # EmbeddingGemma 2: embeddings of the texts seen so far (src/d1.ts:44-46)
        self._lock = threading.Lock()  # one call at a time, as the reference's per-model queue (src/d1.ts:113-119)
        self._pool = cf.ThreadPoolExecutor(max_workers=len(models)) if len(models) > 1 else None

    @staticmethod
    def load(base: str, opts: dict | None = None, *, devices=None, tokensPerPass=None, tokens_per_pass=None,
             **ignored) -> "Decision":
        """A model exported in the reference's format at `base` (a directory holding manifest.json and
        weights.bin), uploaded to every device of `devices` (default [0])."""
        opts = dict(opts or {})
        devices = list(devices if devices is not None else opts.get("devices", [0]))
        if not devices:
            raise DecisionError(_lib.DC_EINVAL, "decision.js: devices is empty")
        if not os.path.exists(os.path.join(base, "manifest.json")):
            raise DecisionError(_lib.DC_EIO, f"decision.js: {base}/manifest.json not found")
        if len(devices) > 1:
            with cf.ThreadPoolExecutor(max_workers=len(devices)) as ex:
                futs = [ex.submit(_Model, base, d) for d in devices]
            errs = [f.exception() for f in futs]
            if any(errs):  # free the replicas that did load, then report the first failure
                for f, e in zip(futs, errs):
                    if e is None:
                        f.result().close()
                raise next(e for e in errs if e is not None)
            models = [f.result() for f in futs]
        else:
            models = [_Model(base, devices[0])]
        kind = models[0].kind
        tpp = tokensPerPass or tokens_per_pass or opts.get("tokensPerPass") or (4096 if kind == "d1-3b" else 8192)
        with open(os.path.join(base, "manifest.json")) as f:
            config = json.load(f).get("config", {})
        tok = None
        if os.path.exists(os.path.join(base, "tokenizer.json")):
            tok = prompts.TextTokenizer.load(base)  # the model's own tokenizer, as src/d1.ts:74 loads it
        workflow = ignored.get("workflow", opts.get("workflow", ""))
        d = Decision(models, kind, int(tpp), config, tok, workflow)
        d.shareState = bool(ignored.get("shareState", opts.get("shareState", False)))
        return d

    def destroy(self):
        """Frees the GPU weights (after a call in flight on another thread has finished); later calls raise."""
        with self._lock:
            for m in self.models:
                m.close()
            self.models = []
            if self._pool:
                self._pool.shutdown()
                self._pool = None

    # ---------------------------------------------------------------- fan-out over devices
    def _fan(self, items, sizes, run_pass, on_progress=None):
        """Runs `items` (whole requests) in passes on every device; returns per-item results in order."""
        with self._lock:
            models = list(self.models)
            n = len(models)
            if n == 0:
                raise DecisionError(_lib.DC_EINVAL, "decision.js: this model was destroyed")
            shards = shard(sizes, n) if n > 1 else [(0, len(items))]
            done = [0]
            lock = threading.Lock()

            def work(w):
                a, b = shards[w]
                res = []
                for i, j in passes(sizes[a:b], self.tokens_per_pass):
                    res.extend(run_pass(models[w], items[a + i:a + j]))
                    if on_progress:
                        with lock:
                            done[0] += j - i
                            on_progress(done[0], len(items))
                return res

            if n == 1:
                return work(0)
            outs = list(self._pool.map(work, range(n)))
        return [r for o in outs for r in o]

    # ---------------------------------------------------------------- engine-level calls
    def embed(self, seqs, on_progress=None):
        """Eg2Engine.embed (src/eg2-engine.ts:72-141): the L2-normalised mean-pooled embedding of every token
        sequence, f32."""
        if self.kind != "eg2":
            raise DecisionError(_lib.DC_EINVAL, f"decision.js: embed needs an encoder model, this is {self.kind}")
        k = [None]

        def run_pass(m, b):
            k[0] = m.embed_dim  # read under _fan's lock, from the replica that ran the pass
            return list(m.encoder_pass(b))

        rows = self._fan(list(seqs), [len(s) for s in seqs], run_pass, on_progress)
        # the reference keeps the first embed_dim values of each pooled row, then normalises
        # (src/eg2-engine.ts:135-139; embed_dim <= embedding_dim, the pooled width)
        k = k[0]
        out = []
        for e in rows:
            e = e[:k] if k else e
            nrm = max(float(np.sqrt((e.astype(np.float64) ** 2).sum())), 1e-12)
            out.append((e / nrm).astype(np.float32))
        return out

    def embed_raw(self, seqs):
        """The pooled embeddings before the host's L2 normalisation (what the GPU computes)."""
        return self._fan(list(seqs), [len(s) for s in seqs], lambda m, b: list(m.encoder_pass(b)))

    def run(self, trees, on_progress=None):
        """D13BEngine.run (src/d1-3b-engine.ts:44-123): option scores [tree][question][option]."""
        if self.kind != "d1-3b":
            raise DecisionError(_lib.DC_EINVAL, f"decision.js: run needs a decoder model, this is {self.kind}")
        sizes = [len(t["trunk"]) + sum(len(b) for b in t["branches"]) for t in trees]
        return self._fan(list(trees), sizes, lambda m, b: m.decoder_pass(b), on_progress)

    # ---------------------------------------------------------------- the System One API
    def _requests_to_trees(self, requests):
        """D13BEngine trees: through the model's tokenizer and d1-3B's prompt (src/d1.ts:195-197), or from tokenized
        requests."""
        trees = []
        for state, qs in requests:
            tokenized = all("branch" in q and "groups" in q for q in qs) and (
                not self.tokenizer or not isinstance(state, str))
            if not tokenized:
                if self.tokenizer is None:
                    raise DecisionError(_lib.DC_EINVAL, "decision.js: this model has no tokenizer.json; a tokenized "
                                        "question needs `branch` (token ids) and `groups` (token ids per option)")
                if self._prompt3b is None:
                    self._prompt3b = prompts.D13BPrompt(self.tokenizer)  # keeps its option-code caches
                p = self._prompt3b
                trees.append({"trunk": p.trunk(state), "branches": [p.branch(q) for q in qs],
                              "groups": [p.readout_ids(q) for q in qs]})
                continue
            trees.append({"trunk": list(state), "branches": [list(q["branch"]) for q in qs],
                          "groups": [[list(g) for g in q["groups"]] for q in qs]})
        return trees

    # ---------------------------------------------------------------- EmbeddingGemma 2 (src/d1.ts:177-214)
    def _remember(self, key, e):
        if len(self._emb) >= 8192:  # the oldest text first
            self._emb.popitem(last=False)
        self._emb[key] = e

    def _eg2_texts(self, state, qs):
        """(state key, [(question key, [option keys])], {key: token ids}) of one request: rendered texts through the
        tokenizer, or the tokenized forms the request carries."""
        seqs = {}
        if all("question_ids" in q and "option_ids" in q for q in qs) and not isinstance(state, str) and (
                isinstance(state, (list, tuple)) and all(isinstance(t, (int, np.integer)) for t in state)):
            sk = ("ids", tuple(int(t) for t in state))
            seqs[sk] = list(sk[1])
            out = []
            for q in qs:
                qk = ("ids", tuple(int(t) for t in q["question_ids"]))
                seqs[qk] = list(qk[1])
                oks = []
                for o in q["option_ids"]:
                    ok = ("ids", tuple(int(t) for t in o))
                    seqs[ok] = list(ok[1])
                    oks.append(ok)
                out.append((qk, oks))
            return sk, out, seqs
        if self.tokenizer is None:
            raise DecisionError(_lib.DC_EINVAL, "decision.js: this model has no tokenizer.json; a tokenized "
                                "EmbeddingGemma 2 request has token-id states and questions with `question_ids` "
                                "and `option_ids`")
        c = self.config
        prompt, max_len = c.get("prompt", ""), int(c.get("max_len", 8192))
        sk = prompts.render_state(state, self.workflow)
        out = []
        for q in qs:
            qt, opts = prompts.render_question(q)
            out.append((qt, opts))
        for t in [sk] + [x for qt, opts in out for x in [qt] + opts]:
            if t not in seqs and t not in self._emb:
                seqs[t] = prompts.tokenize(self.tokenizer, t, prompt, max_len)
        return sk, out, seqs

    def _probs_eg2(self, requests, on_progress=None):
        """Every distinct text (state, question, option) embedded once, then the decision head on the GPU, then
        softmax(logits / temperature) per question, a noul read as [no, yes] and returned as [yes, no]."""
        c = self.config
        types = list(c.get("question_types", ["choice", "score", "noul"]))
        temps = c.get("temperatures", {})
        asked, todo, tokens = [], {}, []
        for state, qs in requests:
            sk, qk, seqs = self._eg2_texts(state, qs)
            asked.append((sk, qk))
            n = 0
            for k, ids in seqs.items():
                if k in self._emb or k in todo:
                    continue
                todo[k] = ids
                n += len(ids)
            tokens.append(n)  # the texts already embedded (a schema after its first use) cost nothing
        keys = list(todo)
        if keys:
            for k, e in zip(keys, self.embed([todo[k] for k in keys], on_progress)):
                self._remember(k, e)
        # the head's inputs: unique states and questions, options per question instance
        srow, qrow, S, Q, O, items, out0 = {}, {}, [], [], [], [], 0
        for (sk, qk), (_, qs) in zip(asked, requests):
            if sk not in srow:
                srow[sk] = len(S)
                S.append(self._emb[sk])
            for (qt, opts), q in zip(qk, qs):
                if q["type"] not in types:
                    raise DecisionError(_lib.DC_EINVAL, f"decision.js: the model has no question type {q['type']}")
                if qt not in qrow:
                    qrow[qt] = len(Q)
                    Q.append(self._emb[qt])
                items.append((srow[sk], qrow[qt], types.index(q["type"]), len(O), len(opts), out0))
                O.extend(self._emb[o] for o in opts)
                out0 += len(opts)
        with self._lock:
            if not self.models:
                raise DecisionError(_lib.DC_EINVAL, "decision.js: this model was destroyed")
            logits = self.models[0].head_logits(np.stack(S), np.stack(Q), np.stack(O),
                                                np.array(items, np.int32).reshape(-1, 6))
        res, i = [], 0
        for (_, qs), n in zip(requests, tokens):
            probs = []
            for q in qs:
                _, _, _, _, no, o0 = items[i]
                t = float(temps.get(q["type"], 1.0))
                p = softmax([float(z) / t for z in logits[o0:o0 + no]])
                probs.append(p[::-1] if q["type"] == "noul" else p)  # the model reads a noul as [no, yes]
                i += 1
            res.append({"probs": probs, "tokens": n})
        return res

    def logits_d3(self, seqs, groups=None, on_progress=None):
        """D3Engine.logits (src/d3-engine.ts:67-139) for (ids, options) sequences: raw code logits per sequence. With
        groups (sequences per request, consecutive) each group shares its common prefix as one trunk."""
        if self.kind != "d3":
            raise DecisionError(_lib.DC_EINVAL, f"decision.js: logits_d3 needs a d3 model, this is {self.kind}")
        groups = list(groups) if groups else [1] * len(seqs)
        items, k = [], 0
        for n in groups:
            items.append(seqs[k:k + n])
            k += n
        sizes = [sum(len(s[0]) for s in it) for it in items]

        def run_pass(m, batch):
            flat = [s for it in batch for s in it]
            out = m.d3_pass(flat, [len(it) for it in batch])
            res, j = [], 0
            for it in batch:
                res.append(out[j:j + len(it)])
                j += len(it)
            return res

        per_item = self._fan(items, sizes, run_pass, on_progress)
        return [x for it in per_item for x in it]

    def _probs_d3(self, requests, on_progress=None):
        """Decision.runD3 (src/d1.ts:149-169): one sequence per question, through the model's tokenizer and d3-lite's
        prompt (or tokenized: a question holding `ids` and `options`), softmax of the code logits over the
        temperature, a noul read as [false, true] and returned as [true, false]."""
        codes = self.config.get("codes") or []
        temp = float(self.config.get("temperature", 1.0) or 1.0)
        seqs, groups = [], []
        for state, qs in requests:
            for q in qs:
                if "ids" in q and "options" in q:
                    seqs.append((list(q["ids"]), int(q["options"])))
                else:
                    if self.tokenizer is None:
                        raise DecisionError(_lib.DC_EINVAL, "decision.js: this model has no tokenizer.json; a "
                                            "tokenized d3 question needs `ids` and `options`")
                    try:
                        seqs.append(prompts.d3_encode(self.tokenizer, state, q, codes))
                    except ValueError as e:
                        raise DecisionError(_lib.DC_EINVAL, str(e)) from None
                if seqs[-1][1] > len(codes):
                    raise DecisionError(_lib.DC_EINVAL, f"decision.js: d3 reads {len(codes)} codes, a question has "
                                        f"{seqs[-1][1]} options")
            groups.append(len(qs))
        logits = self.logits_d3(seqs, groups if self.shareState else None, on_progress) if seqs else []
        out, k = [], 0
        for (state, qs), n in zip(requests, groups):
            probs = []
            for q in qs:
                p = softmax([float(z) / temp for z in logits[k]])
                probs.append(p[::-1] if q.get("type") == "noul" else p)
                k += 1
            out.append({"probs": probs, "tokens": sum(len(s[0]) for s in seqs[k - n:k])})
        return out

    def logits_omni(self, seqs, on_progress=None):
        """D1OmniEngine.logits (src/omni-engine.ts:56-141) for (ids, markers, type) sequences: raw logits at the
        option markers, per sequence."""
        if self.kind not in ("d1-omni", "laya"):
            raise DecisionError(_lib.DC_EINVAL, f"decision.js: logits_omni needs a d1-omni or Laya model, this is "
                                f"{self.kind}")
        run = (lambda m, b: m.laya_pass(b)) if self.kind == "laya" else (lambda m, b: m.omni_pass(b))
        return self._fan(list(seqs), [len(s[0]) for s in seqs], run, on_progress)

    def _probs_omni(self, requests, on_progress=None):
        """Decision.runEncoder for d1-omni and Laya (src/d1.ts:121-147): one sequence per question (through the model's
        tokenizer and prompt, or tokenized: a question holding `ids` and `markers`), softmax of the marker logits
        over the question's calibrated temperature, a noul read as [false, true] and returned as [true, false]."""
        temps = self.config.get("temperatures") or {}
        laya = self.kind == "laya"
        max_len = int(self.config.get("max_len" if laya else "max_length", 512 if laya else 16384))
        head_max_len = int(self.config.get("head_max_len", 192))
        seqs, counts = [], []
        for state, qs in requests:
            for q in qs:
                if "ids" in q and "markers" in q:
                    ids, mk = list(q["ids"]), list(q["markers"])
                else:
                    if self.tokenizer is None:
                        raise DecisionError(_lib.DC_EINVAL, "decision.js: this model has no tokenizer.json; a "
                                            "tokenized d1-omni question needs `ids` and `markers`")
                    try:
                        ids, mk = (prompts.laya_encode(self.tokenizer, state, q, max_len, head_max_len) if laya
                                   else prompts.omni_encode(self.tokenizer, state, q, max_len))
                    except ValueError as e:
                        raise DecisionError(_lib.DC_EINVAL, str(e)) from None
                seqs.append((ids, mk, OMNI_TYPES[q["type"]]))
            counts.append(len(qs))
        logits = self.logits_omni(seqs, on_progress) if seqs else []
        out, k = [], 0
        for (state, qs), n in zip(requests, counts):
            probs = []
            for q in qs:
                t = float(temps.get(prompts.omni_temperature_key(q), temps.get(q["type"], 1.0)) or 1.0)
                p = softmax([float(z) / t for z in logits[k]])
                probs.append(p[::-1] if q["type"] == "noul" else p)
                k += 1
            out.append({"probs": probs, "tokens": sum(len(s[0]) for s in seqs[k - n:k])})
        return out

    def _probs(self, requests, on_progress=None):
        for _, qs in requests:
            for q in qs:
                check_question(q)
        if self.kind in ("d1-omni", "laya"):
            return self._probs_omni(requests, on_progress)
        if self.kind == "eg2":
            return self._probs_eg2(requests, on_progress)
        if self.kind == "d3":
            return self._probs_d3(requests, on_progress)
        if self.kind != "d1-3b":
            raise DecisionError(_lib.DC_EINVAL, f"decision.js: typed decisions need a d1-3b, d1-omni, Laya, d3 or eg2 model, "
                                f"this is {self.kind}")
        trees = self._requests_to_trees(requests)
        scores = self.run(trees, on_progress)
        out = []
        for tr, per_q in zip(trees, scores):
            tokens = len(tr["trunk"]) + sum(len(b) for b in tr["branches"])
            out.append({"probs": [softmax(s) for s in per_q], "tokens": tokens})
        return out

    def systemOne(self, state, questions: dict) -> dict:
        """Named questions over one state, in one call (src/d1.ts:82-84)."""
        return self.systemOneBatch([[state, questions]])[0]

    def systemOneBatch(self, requests, opts: dict | None = None) -> list:
        """Many [state, {name: question}] requests, packed into as few forward passes as fit (src/d1.ts:87-95)."""
        on_progress = (opts or {}).get("onProgress")
        done = self._probs([[s, list(qs.values())] for s, qs in requests], on_progress)
        legend = str if self.kind == "d1-3b" else prompts.criterion  # src/d1.ts:89
        res = []
        for (s, qs), d in zip(requests, done):
            names = list(qs.keys())
            res.append({"answers": {n: answer(qs[n], d["probs"][j], legend) for j, n in enumerate(names)},
                        "usage": {"input_tokens": d["tokens"], "output_tokens": 0}})
        return res

    def probabilities(self, state, questions) -> list:
        """Each question's distribution over its options (src/d1.ts:98-100)."""
        return self._probs([[state, list(questions)]])[0]["probs"]

    def probabilitiesBatch(self, requests, opts: dict | None = None) -> list:
        """probabilities for many [state, questions] requests (src/d1.ts:103-105)."""
        return [d["probs"] for d in self._probs([[s, list(q)] for s, q in requests], (opts or {}).get("onProgress"))]
