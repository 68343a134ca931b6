"""Seeded synthetic workloads with the shapes and value distributions of the
benchmark configurations (no dataset is involved; all inputs are generated).

  C0  1 row fp32, T 0.7, top_k 20, top_p 0.8, repeat 1.05 over 256 tokens
  C1  64 rows fp32, T 0.6, top_k 20, top_p 0.95, penalties 1.1/0.5/0.3,
      1,024-token histories
  C2  256 rows bf16, per-row parameters (10% greedy, top_k in {0,20,50,100},
      top_p U[0.5,1], min_p in {0,.05,.1}, histories U[0,8192])
  C3  MTP verify, 32 sequences x (3 drafts + bonus), T 0.8, top_p 0.9
  C4  1,024 rows bf16, top_k 50, top_p 0.9, T 1.0, repeat 1.1 over 4,096
Logits: C0/C1/C4 are 2.5*N(0,1) plus a Zipf(s=1.1) bias (-1.1*ln(rank))
placed on a seeded random permutation of the ids; C2 is 3*N(0,1) plus a +8
spike on 1-3 random ids per row; C3 drafts are target + 0.5*N(0,1).
Uniforms are Philox4x32-10 draws quantised to the 2^-24 grid.
"""
from __future__ import annotations

import zlib
from dataclasses import dataclass
from typing import Optional

import numpy as np

from .params import HAS_MIN_P, PARAMS_DTYPE

V_DEFAULT = 151_936


# ---- Philox4x32-10 (Salmon et al., SC'11) ----------------------------------
_M0, _M1 = np.uint64(0xD2511F53), np.uint64(0xCD9E8D57)
_W0, _W1 = np.uint32(0x9E3779B9), np.uint32(0xBB67AE85)


def philox4x32(counter: np.ndarray, key: np.ndarray, rounds: int = 10) -> np.ndarray:
    """counter: (n, 4) uint32, key: (n, 2) uint32 -> (n, 4) uint32."""
    c = counter.astype(np.uint32).copy()
    k0 = key[:, 0].astype(np.uint32).copy()
    k1 = key[:, 1].astype(np.uint32).copy()
    for _ in range(rounds):
        p0 = c[:, 0].astype(np.uint64) * _M0
        p1 = c[:, 2].astype(np.uint64) * _M1
        hi0 = (p0 >> np.uint64(32)).astype(np.uint32)
        lo0 = (p0 & np.uint64(0xFFFFFFFF)).astype(np.uint32)
        hi1 = (p1 >> np.uint64(32)).astype(np.uint32)
        lo1 = (p1 & np.uint64(0xFFFFFFFF)).astype(np.uint32)
        c = np.stack([hi1 ^ c[:, 1] ^ k0, lo1, hi0 ^ c[:, 3] ^ k1, lo0], axis=1)
        k0 = (k0 + _W0).astype(np.uint32)
        k1 = (k1 + _W1).astype(np.uint32)
    return c


def philox_uniforms(seed: int, n: int, stream: int = 0) -> np.ndarray:
    """n uniforms in [0, 1) on the 2^-24 grid: (x0 >> 8) * 2^-24 of block i."""
    idx = np.arange(n, dtype=np.uint64)
    ctr = np.zeros((n, 4), np.uint32)
    ctr[:, 0] = (idx & np.uint64(0xFFFFFFFF)).astype(np.uint32)
    ctr[:, 1] = (idx >> np.uint64(32)).astype(np.uint32)
    ctr[:, 2] = np.uint32(stream & 0xFFFFFFFF)
    key = np.zeros((n, 2), np.uint32)
    key[:, 0] = np.uint32(seed & 0xFFFFFFFF)
    key[:, 1] = np.uint32((seed >> 32) & 0xFFFFFFFF)
    x = philox4x32(ctr, key)[:, 0]
    return ((x >> np.uint32(8)).astype(np.float64) * 2.0**-24).astype(np.float32)


# ---- logits ------------------------------------------------------------------
def zipf_logits(rng: np.random.Generator, rows: int, vocab: int, sigma: float = 2.5,
                s: float = 1.1) -> np.ndarray:
    ranks = np.arange(1, vocab + 1, dtype=np.float64)
    bias = (-s * np.log(ranks)).astype(np.float32)
    out = np.empty((rows, vocab), np.float32)
    for r in range(rows):
        perm = rng.permutation(vocab)
        out[r, perm] = bias
        out[r] += (sigma * rng.standard_normal(vocab)).astype(np.float32)
    return out


def spike_logits(rng: np.random.Generator, rows: int, vocab: int) -> np.ndarray:
    out = (3.0 * rng.standard_normal((rows, vocab))).astype(np.float32)
    for r in range(rows):
        m = int(rng.integers(1, 4))
        out[r, rng.choice(vocab, size=m, replace=False)] += 8.0
    return out


def to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even f32 -> bf16, returned as uint16 bits."""
    b = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    nan = np.isnan(x)
    r = ((b + np.uint64(0x7FFF) + ((b >> np.uint64(16)) & np.uint64(1))) >> np.uint64(16)).astype(np.uint16)
    r[nan] = np.uint16(0x7FC0)
    return r


def bf16_bits_to_f32(h: np.ndarray) -> np.ndarray:
    return (h.astype(np.uint32) << np.uint32(16)).view(np.float32)


def params_rows(rows: int, temperature: float, top_p: float = 1.0, top_k: int = 0,
                min_p: Optional[float] = None, repeat_penalty: float = 1.0,
                repeat_last_n: int = 64, frequency_penalty: float = 0.0,
                presence_penalty: float = 0.0) -> np.ndarray:
    p = np.zeros(rows, PARAMS_DTYPE)
    p["temperature"] = temperature
    p["top_p"] = top_p
    p["top_k"] = top_k
    p["min_p"] = 0.0 if min_p is None else min_p
    p["flags"] = 0 if min_p is None else HAS_MIN_P
    p["repeat_penalty"] = repeat_penalty
    p["repeat_last_n"] = repeat_last_n
    p["frequency_penalty"] = frequency_penalty
    p["presence_penalty"] = presence_penalty
    return p


@dataclass
class Batch:
    name: str
    logits: np.ndarray        # rows x vocab, float32 or uint16 (bf16 bits)
    params: np.ndarray        # rows PARAMS_DTYPE
    hist: np.ndarray          # int32 concatenated histories
    hist_off: np.ndarray      # int64 rows+1
    uniforms: np.ndarray      # float32 rows
    dtype: str                # "f32" | "bf16"

    @property
    def rows(self) -> int:
        return self.logits.shape[0]

    @property
    def vocab(self) -> int:
        return self.logits.shape[1]

    def logits_f32(self) -> np.ndarray:
        return self.logits if self.dtype == "f32" else bf16_bits_to_f32(self.logits)

    def algorithmic_bytes(self) -> int:
        """Logits + history read once (the roofline numerator)."""
        esz = 4 if self.dtype == "f32" else 2
        return self.rows * self.vocab * esz + 4 * int(self.hist_off[-1])


def _histories(rng, lengths, vocab):
    off = np.zeros(len(lengths) + 1, np.int64)
    off[1:] = np.cumsum(lengths)
    hist = rng.integers(0, vocab, size=int(off[-1]), dtype=np.int64).astype(np.int32)
    return hist, off


def config(name: str, rows: Optional[int] = None, vocab: int = V_DEFAULT, seed: int = 0) -> Batch:
    rng = np.random.default_rng([seed, zlib.crc32(name.encode())])
    if name in ("c0", "c1", "c1x256"):
        if name == "c0":
            n = rows or 1
            hlen, params = 256, params_rows(n, 0.7, top_p=0.8, top_k=20, repeat_penalty=1.05,
                                             repeat_last_n=256)
        else:
            n = rows or (64 if name == "c1" else 256)
            hlen, params = 1024, params_rows(n, 0.6, top_p=0.95, top_k=20, repeat_penalty=1.1,
                                              repeat_last_n=1024, presence_penalty=0.5,
                                              frequency_penalty=0.3)
        logits = zipf_logits(rng, n, vocab)
        hist, off = _histories(rng, [hlen] * n, vocab)
        return Batch(name, logits, params, hist, off, philox_uniforms(seed + 1, n), "f32")
    if name == "c2":
        n = rows or 256
        p = np.zeros(n, PARAMS_DTYPE)
        p["temperature"] = rng.uniform(0.1, 1.5, n).astype(np.float32)
        greedy = rng.random(n) < 0.10
        p["temperature"][greedy] = 0.0
        p["top_k"] = rng.choice([0, 20, 50, 100], n)
        p["top_p"] = rng.uniform(0.5, 1.0, n).astype(np.float32)
        mp = rng.choice([0.0, 0.05, 0.1], n)
        p["min_p"] = mp
        p["flags"] = np.where(mp > 0, HAS_MIN_P, 0)
        p["repeat_penalty"] = rng.uniform(1.0, 1.3, n).astype(np.float32)
        p["frequency_penalty"] = rng.uniform(0.0, 0.5, n).astype(np.float32)
        p["presence_penalty"] = rng.uniform(0.0, 0.5, n).astype(np.float32)
        lengths = rng.integers(0, 8193, n)
        p["repeat_last_n"] = lengths
        logits = to_bf16_bits(spike_logits(rng, n, vocab))
        hist, off = _histories(rng, lengths, vocab)
        return Batch(name, logits, p, hist, off, philox_uniforms(seed + 2, n), "bf16")
    if name == "c4":
        n = rows or 1024
        params = params_rows(n, 1.0, top_p=0.9, top_k=50, repeat_penalty=1.1, repeat_last_n=4096)
        logits = to_bf16_bits(zipf_logits(rng, n, vocab))
        hist, off = _histories(rng, [4096] * n, vocab)
        return Batch(name, logits, params, hist, off, philox_uniforms(seed + 4, n), "bf16")
    raise ValueError(f"unknown config {name}")


@dataclass
class MtpBatch:
    """Configuration 3: MTP verify inputs. target: seqs x (L+1) x vocab,
    draft: seqs x L x vocab (f32), drafts: seqs x L, uniforms: seqs x (L+1)."""

    name: str
    target: np.ndarray
    draft: np.ndarray
    drafts: np.ndarray
    params: np.ndarray
    uniforms: np.ndarray

    @property
    def seqs(self) -> int:
        return self.target.shape[0]

    @property
    def draft_len(self) -> int:
        return self.draft.shape[1]

    def algorithmic_bytes(self) -> int:
        """Target and draft logits read once."""
        return int(self.target.nbytes + self.draft.nbytes)


def mtp_config(seqs: int = 32, draft_len: int = 3, vocab: int = V_DEFAULT, seed: int = 0,
               temperature: float = 0.8, top_p: float = 0.9, top_k: int = 0) -> MtpBatch:
    """Target logits as configuration 0 (2.5 N(0,1) + Zipf bias), draft =
    target + 0.5 N(0,1). Draft tokens are drawn from the draft's softmax at
    `temperature` over its 256 largest logits with seeded uniforms (input
    generation, not the sampler under test)."""
    rng = np.random.default_rng([seed, zlib.crc32(b"c3")])
    rows = seqs * (draft_len + 1)
    target = zipf_logits(rng, rows, vocab).reshape(seqs, draft_len + 1, vocab)
    draft = (target[:, :draft_len, :] + 0.5 * rng.standard_normal((seqs, draft_len, vocab))).astype(np.float32)
    drafts = np.zeros((seqs, draft_len), np.int32)
    for s in range(seqs):
        for j in range(draft_len):
            row = draft[s, j]
            top = np.argpartition(row, -256)[-256:]
            z = row[top].astype(np.float64) / max(temperature, 1e-3)
            w = np.exp(z - z.max())
            drafts[s, j] = int(rng.choice(top, p=w / w.sum()))
    params = params_rows(seqs, temperature, top_p=top_p, top_k=top_k)
    u = philox_uniforms(seed + 3, seqs * (draft_len + 1)).reshape(seqs, draft_len + 1)
    return MtpBatch("c3", target, draft, drafts, params, u)
