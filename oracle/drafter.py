"""numpy restatement of the per-token drafter (test oracle; see ``oracle/__init__.py``).

Follows ``RefDrafter`` (``drafting/cpu_drafter.py:76-289``), the reference's PyTorch
restatement of the C++ drafter (``drafting/cpu/drafter.cpp:396-556``).  Inputs are the
bundle arrays of ``drafting/export_drafter.py:25-34`` (as numpy arrays, tables fp16/fp32).
The SSM variant (SD-C) is restated too (``cpu_drafter.py:160-166``).
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np

F32 = np.float32


def _rms(x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    """``cpu_drafter.py:60-61``: x * rsqrt(mean(x^2) + eps) * w (fp32)."""
    x = x.astype(F32)
    ms = np.mean(np.square(x, dtype=F32), axis=-1, keepdims=True, dtype=F32)
    return (x * (F32(1.0) / np.sqrt(ms + F32(eps))) * w.astype(F32)).astype(F32)


@dataclass(frozen=True)
class Cursor:
    """``cpu_drafter.py:64-69``: position of the last processed token, that token, SSM state,
    codes of the last max(ngrams) positions (oldest first)."""

    t: int
    tok: int
    s: np.ndarray | None
    hist: tuple


@dataclass
class DraftOut:
    tokens: list
    topk_ids: np.ndarray
    topk_logits: np.ndarray
    codes: np.ndarray


class OracleDrafter:
    """Stateful drafter with the ``RefDrafter`` API: reset / length / truncate / committed_codes /
    commit / draft / trace."""

    def __init__(self, config: dict, arrays: dict, topk: int = 3, shortlist_cap: int | None = None):
        c = self.cfg = dict(config)
        self.topk = int(topk)
        self.ngrams = [int(n) for n in c["ngrams"]]
        self.maxn = max(self.ngrams)
        self.R, self.bits, self.V = int(c["routes"]), int(c["bits"]), int(c["vocab"])
        self.kv, self.hd, self.G = int(c["kv_heads"]), int(c["head_dim"]), int(c["groups"])
        a = {k: np.asarray(v) for k, v in arrays.items()}
        self.E = a["embedding"].astype(F32)
        self.tables = {n: a[f"table_{n}"] for n in self.ngrams}
        self.mem_norm, self.kv_proj = a["mem_norm"].astype(F32), a["kv_proj"].astype(F32)
        self.router = a["router"].astype(F32)
        self.prev_norm, self.cur_norm, self.start = a["router_prev_norm"], a["router_cur_norm"], a["router_start"]
        self.has_ssm = "ssm_w_in" in a
        if self.has_ssm:
            self.ssm_norm, self.ssm_w_in, self.ssm_a = a["ssm_norm"], a["ssm_w_in"].astype(F32), a["ssm_decay"].astype(F32)
        self.router_ssm = c["router_kind"] == "embed2_ssm"
        self.q_norm, self.w_q, self.w_o, self.out_norm = a["q_norm"], a["w_q"].astype(F32), a["w_o"].astype(F32), a["out_norm"]
        self.w_sq = a.get("w_sq")
        self.sk_ids = {n: a[f"sketch_ids_{n}"] for n in self.ngrams if f"sketch_ids_{n}" in a}
        self.sk_cnt = {n: a[f"sketch_counts_{n}"] for n in self.ngrams if n in self.sk_ids}
        self.fallback = [int(x) for x in a.get("fallback", np.zeros(0, np.int32))]
        self.cap = int(c["shortlist_cap"] if shortlist_cap is None else shortlist_cap)
        self.reset()

    # ------------------------------------------------------------------ state (``:123-155``)
    def reset(self) -> None:
        self._tokens: list = []
        self._codes: list = []
        self._ssm: list = []

    @property
    def length(self) -> int:
        return len(self._tokens)

    @property
    def tokens(self) -> list:
        return list(self._tokens)

    def committed_codes(self) -> np.ndarray:
        return np.stack(self._codes) if self._codes else np.zeros((0, self.R), np.uint8)

    def truncate(self, length: int) -> None:
        if not 0 <= length <= self.length:
            raise ValueError(f"cannot truncate to {length} (length {self.length})")
        del self._tokens[length:], self._codes[length:], self._ssm[length:]

    def commit(self, tokens, codes=None) -> None:
        cur = self._cursor()
        for i, tok in enumerate(tokens):
            cur = self.advance(cur, int(tok), None if codes is None else np.asarray(codes[i], np.uint8))
            self._tokens.append(int(tok))
            self._codes.append(cur.hist[-1])
            self._ssm.append(cur.s)

    def _cursor(self) -> Cursor:
        n = self.length
        if n == 0:
            return Cursor(-1, -1, None, ())
        return Cursor(n - 1, self._tokens[-1], self._ssm[-1], tuple(self._codes[max(0, n - self.maxn):]))

    # ------------------------------------------------------------------ per token (``:158-210``)
    def advance(self, cur: Cursor, tok: int, code: np.ndarray | None = None) -> Cursor:
        """``cpu_drafter.py:158-176``: SSM step, embed2 router -> sign codes, history shift."""
        if not 0 <= tok < self.V:
            raise ValueError("token id out of range")
        e = self.E[tok]
        s = None
        if self.has_ssm:
            u = self.ssm_w_in @ _rms(e, self.ssm_norm, self.cfg["ssm_eps"])
            prev = cur.s if cur.s is not None else np.zeros_like(u)
            s = (self.ssm_a * prev + (F32(1) - self.ssm_a) * u).astype(F32)
        if code is None:
            ep = self.E[cur.tok] if cur.t >= 0 else self.start
            eps = self.cfg["router_eps"]
            parts = [_rms(ep, self.prev_norm, eps), _rms(e, self.cur_norm, eps)]
            if self.router_ssm:
                parts.append(s)
            logits = (self.router @ np.concatenate(parts)).astype(F32)
            bits = (logits > 0).reshape(self.R, self.bits).astype(np.int64)
            code = (bits << np.arange(self.bits)).sum(-1).astype(np.uint8)
        return Cursor(cur.t + 1, tok, s, (cur.hist + (np.asarray(code, np.uint8),))[-self.maxn:])

    def rows(self, cur: Cursor) -> dict:
        """``cpu_drafter.py:178-189``: v2 rows r * A**n + sum_k c[t-n+1+k] << (k*bits), None if t < n-1."""
        out = {}
        r = np.arange(self.R, dtype=np.int64)
        for n in self.ngrams:
            if cur.t < n - 1:
                out[n] = None
                continue
            addr = np.zeros(self.R, np.int64)
            for k in range(n):
                addr |= cur.hist[len(cur.hist) - n + k].astype(np.int64) << (k * self.bits)
            out[n] = r * (1 << self.bits) ** n + addr
        return out

    def shortlist(self, rows: dict) -> np.ndarray | None:
        """``cpu_drafter.py:191-217``: sketch counts summed per token, (count desc, id asc), cap,
        then fallback tokens; None means full vocabulary."""
        if self.cap <= 0 or not self.sk_ids:
            return None
        ids, cnt = [], []
        for n in self.ngrams:
            if rows[n] is None:
                continue
            ids.append(np.asarray(self.sk_ids[n][rows[n]], np.int64).ravel())
            cnt.append(np.asarray(self.sk_cnt[n][rows[n]], np.int64).ravel())
        out: list = []
        if ids:
            i, c = np.concatenate(ids), np.concatenate(cnt)
            i, c = i[c > 0], c[c > 0]
            if len(i):
                uniq, inv = np.unique(i, return_inverse=True)
                tot = np.zeros(len(uniq), np.int64)
                np.add.at(tot, inv, c)
                order = np.lexsort((uniq, -tot))[: self.cap]
                out = [int(x) for x in uniq[order]]
        if len(out) < self.cap and self.fallback:
            have = set(out)
            for f in self.fallback:
                if len(out) >= self.cap:
                    break
                if f not in have:
                    out.append(f)
                    have.add(f)
        return np.asarray(out, np.int64) if out else None

    def hidden(self, cur: Cursor, rows: dict | None = None) -> np.ndarray:
        """``cpu_drafter.py:219-239`` (= ``DraftReadout.hidden``): rows -> memory RMSNorm -> KV;
        query W_q RMSNorm(e) (+ W_sq s); sink attention over routes; W_o -> RMSNorm."""
        rows = self.rows(cur) if rows is None else rows
        c = self.cfg
        mem_dim = int(c["mem_dim"])
        parts = []
        for n in self.ngrams:
            if rows[n] is None:
                parts.append(np.zeros((self.R, mem_dim), F32))
            else:
                parts.append(np.asarray(self.tables[n][rows[n]]).astype(F32))
        tok = np.concatenate(parts, -1)
        kv = _rms(tok, self.mem_norm, c["mem_eps"]) @ self.kv_proj.T
        kh = self.kv * self.hd
        key = kv[:, :kh].reshape(self.R, self.kv, self.hd).transpose(1, 0, 2)
        val = kv[:, kh:].reshape(self.R, self.kv, self.hd).transpose(1, 0, 2)
        q = self.w_q @ _rms(self.E[cur.tok], self.q_norm, c["draft_eps"])
        if self.w_sq is not None:
            q = q + np.asarray(self.w_sq, F32) @ cur.s
        q = q.astype(F32).reshape(self.kv, self.G, self.hd)
        scores = (q @ np.swapaxes(key, -1, -2)).astype(F32) * F32(c["softmax_scale"])
        sink = F32(c["sink_logit"])
        mx = np.maximum(scores.max(-1, keepdims=True), sink)
        ex = np.exp(scores - mx).astype(F32)
        probs = ex / (ex.sum(-1, keepdims=True, dtype=F32) + np.exp(sink - mx))
        out = (probs.astype(F32) @ val).astype(F32).reshape(-1)
        return _rms(self.w_o @ out, self.out_norm, c["draft_eps"])

    def readout(self, cur: Cursor, full: bool = False) -> tuple[np.ndarray, np.ndarray]:
        """``cpu_drafter.py:241-248``: (candidate ids, logits E[ids] . h)."""
        rows = self.rows(cur)
        h = self.hidden(cur, rows)
        sl = None if full else self.shortlist(rows)
        if sl is None:
            return np.arange(self.V, dtype=np.int64), (self.E @ h).astype(F32)
        return sl, (self.E[sl] @ h).astype(F32)

    @staticmethod
    def top_order(logits: np.ndarray, k: int) -> np.ndarray:
        """Top-k by (logit desc, index asc): ``cpu_drafter.py:263`` stable descending sort,
        ``drafter.cpp:547-556``."""
        return np.lexsort((np.arange(len(logits)), -logits.astype(np.float64)))[:k]

    # ------------------------------------------------------------------ API (``:251-289``)
    def draft(self, gamma: int, hyp=(), topk: int | None = None, last_codes: bool = False) -> DraftOut:
        k = int(topk or self.topk)
        cur = self._cursor()
        if cur.t < 0 and not len(hyp):
            raise ValueError("draft needs at least one committed or hypothetical token")
        codes = []
        for tok in hyp:
            cur = self.advance(cur, int(tok))
            codes.append(cur.hist[-1])
        ids = np.full((gamma, k), -1, np.int64)
        lg = np.full((gamma, k), -np.inf, np.float32)
        toks = []
        for i in range(gamma):
            sl, logits = self.readout(cur)
            order = self.top_order(logits, k)
            ids[i, :len(order)] = sl[order]
            lg[i, :len(order)] = logits[order]
            toks.append(int(ids[i, 0]))
            if i + 1 < gamma or last_codes:
                cur = self.advance(cur, toks[-1])
                codes.append(cur.hist[-1])
        return DraftOut(toks, ids, lg, np.stack(codes) if codes else np.zeros((0, self.R), np.uint8))

    def trace(self, tokens, codes=None, full: bool = False) -> tuple[np.ndarray, np.ndarray, np.ndarray]:
        """``cpu_drafter.py:272-289``: teacher-forced pass from an empty state."""
        tokens = [int(x) for x in tokens]
        full_vocab = full or self.cap <= 0 or not self.sk_ids
        s_dim = self.V if full_vocab else self.cap
        n = len(tokens)
        out_c = np.zeros((n, self.R), np.uint8)
        out_i = np.full((n, s_dim), -1, np.int64)
        out_l = np.full((n, s_dim), -np.inf, np.float32)
        cur = Cursor(-1, -1, None, ())
        for t, tok in enumerate(tokens):
            cur = self.advance(cur, tok, None if codes is None else np.asarray(codes[t], np.uint8))
            out_c[t] = cur.hist[-1]
            sl, lg = self.readout(cur, full)
            m = min(len(sl), s_dim)
            out_i[t, :m], out_l[t, :m] = sl[:m], lg[:m]
        return out_c, out_i, out_l


# ------------------------------------------------------------------ online counts (acceptance harness)
def ngram_rows_seq(codes: np.ndarray, order: int, bits: int) -> np.ndarray:
    """``drafting/build_sketches.py:186-197`` (``seq_rows``) for one record: rows [T, R] of the n-grams
    ending at each t (oldest code least significant, route offset r * 2^(bits order)); -1 for t < order-1."""
    T, R = codes.shape
    c = codes.astype(np.int64)
    out = np.full((T, R), -1, np.int64)
    if T >= order:
        addr = c[: T - order + 1].copy()
        for e in range(1, order):
            addr |= c[e: e + T - order + 1] << (e * bits)
        out[order - 1:] = np.arange(R, dtype=np.int64) * (1 << (bits * order)) + addr
    return out


def ngram_rows_window(win: np.ndarray, real: np.ndarray, order: int, bits: int) -> np.ndarray:
    """``drafting/drafters.py:99-107`` (``window_rows``): rows [N, R] of the n-gram ending at each window's
    last slot, -1 unless its last ``order`` slots are all real."""
    N, W, R = win.shape
    c = win[:, W - order:].astype(np.int64)
    addr = c[:, 0].copy()
    for e in range(1, order):
        addr |= c[:, e] << (e * bits)
    rows = np.arange(R, dtype=np.int64) * (1 << (bits * order)) + addr
    ok = real[:, W - order:].all(1)
    return np.where(ok[:, None], rows, -1)


def online_counts_mix(codes, x, orders, bits: int, vocab: int, kappa: float, p, win, real, deadline) -> np.ndarray:
    """``drafting/drafters.py:117-143`` (``OnlineCounts(codes, x, ...).mix(p, win, real, deadline)``): the
    record's verified pairs (t, x[t+1]) vote for x[t+1] with weight w[j, t] = the (order, route) rows that
    pair t shares with query window j (pairs t <= deadline[j] only); the votes' distribution is mixed
    into p with lambda = n_eff / (n_eff + kappa), n_eff = sum_t w / (R x orders), in the reference's
    fp32 operation order."""
    codes = np.asarray(codes)
    T, R = codes.shape
    nxt = np.asarray(x, np.int64)[1:]
    p = np.asarray(p, F32)
    N = p.shape[0]
    w = np.zeros((N, T - 1), F32)
    for n in orders:
        keys = ngram_rows_seq(codes, n, bits)[:-1]                       # pairs t = 0 .. T-2
        q = ngram_rows_window(np.asarray(win), np.asarray(real, bool), n, bits)
        w += ((keys[None] == q[:, None]) & (q[:, None] >= 0)).sum(-1).astype(F32)
    w = w * (np.arange(T - 1)[None] <= np.asarray(deadline)[:, None]).astype(F32)
    tot = w.sum(1, keepdims=True, dtype=F32)
    sc = np.zeros((N, vocab), F32)
    for j in range(N):
        np.add.at(sc[j], nxt, w[j])
    n_eff = (tot / F32(R * len(orders))).astype(F32)
    lam = (n_eff / (n_eff + F32(kappa))).astype(F32)
    return ((F32(1) - lam) * p + (lam * sc) / np.maximum(tot, F32(1e-9))).astype(F32)
