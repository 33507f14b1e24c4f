"""Seeded synthetic GGUF super-blocks and qwen3moe GGUF files.

Data formats follow the GGUF/ggml layouts the reference decodes (qwen3moe.cpp:69-218 for the blocks,
qwen3moe.cpp:285-347 for the file): a block's bytes are random except the fp16 scale fields, which are
set from the distribution a configuration names, so every encodable scale/min/nibble pattern occurs.

Every tensor is generated from its own seed sequence ``(seed, tensor index, chunk index)`` in fixed-size
chunks, so the bytes do not depend on the order or the process that generates them: the GPU arm, the
reference arm and the tests regenerate identical models independently.
"""
from __future__ import annotations

import dataclasses
import hashlib
import os
import struct
from typing import Callable, Iterable

import numpy as np

# ggml type id -> (elements per block, bytes per block)   (qwen3moe.cpp:204-218)
BLOCK = {0: (32, 128), 1: (32, 64), 8: (32, 34), 12: (256, 144), 13: (256, 176), 14: (256, 210)}
F32, F16, Q8_0, Q4_K, Q5_K, Q6_K = 0, 1, 8, 12, 13, 14
TYPE_NAME = {0: "F32", 1: "F16", 8: "Q8_0", 12: "Q4_K", 13: "Q5_K", 14: "Q6_K"}

CHUNK_BLOCKS = 1 << 18  # blocks per generation chunk (36-55 MiB for the K-quants)


def row_bytes(qtype: int, ne0: int) -> int:
    blck, nb = BLOCK[qtype]
    assert ne0 % blck == 0, (qtype, ne0)
    return ne0 // blck * nb


def _rng(*key: int) -> np.random.Generator:
    return np.random.Generator(np.random.PCG64(np.random.SeedSequence([int(k) & 0xFFFFFFFF for k in key])))


def _random_bytes(rng: np.random.Generator, n: int) -> np.ndarray:
    words = rng.bit_generator.random_raw((n + 7) // 8)
    return words.view(np.uint8)[:n]


def _f16_bytes(v: np.ndarray) -> np.ndarray:
    return v.astype(np.float16).view(np.uint8).reshape(-1, 2)


def quant_blocks(qtype: int, nblocks: int, rng: np.random.Generator, d_sigma: float) -> np.ndarray:
    """``nblocks`` random blocks of ``qtype`` as a (nblocks, block bytes) uint8 array.

    Q4_K/Q5_K: fp16 d and dmin ~ |N(0, d_sigma)|; the 12 scale bytes, the high-bit plane and the nibbles
    are uniform bytes, so the 6-bit scales/mins are uniform 0..63.
    Q6_K: ql/qh uniform bytes, int8 sub-scales uniform -32..31, fp16 d ~ |N(0, d_sigma)| at byte 208.
    Q8_0: int8 quants uniform, fp16 d ~ |N(0, d_sigma)|.
    """
    blck, nb = BLOCK[qtype]
    raw = _random_bytes(rng, nblocks * nb).reshape(nblocks, nb)  # a fresh, writable buffer
    if qtype in (Q4_K, Q5_K):
        raw[:, 0:2] = _f16_bytes(np.abs(rng.normal(0.0, d_sigma, nblocks)))
        raw[:, 2:4] = _f16_bytes(np.abs(rng.normal(0.0, d_sigma, nblocks)))
    elif qtype == Q6_K:
        raw[:, 192:208] = rng.integers(-32, 32, size=(nblocks, 16), dtype=np.int8).view(np.uint8)
        raw[:, 208:210] = _f16_bytes(np.abs(rng.normal(0.0, d_sigma, nblocks)))
    elif qtype == Q8_0:
        raw[:, 0:2] = _f16_bytes(np.abs(rng.normal(0.0, d_sigma, nblocks)))
    else:
        raise ValueError(f"quant_blocks: type {qtype} is not a block-quantized type")
    return raw


@dataclasses.dataclass
class TensorSpec:
    name: str
    qtype: int
    shape: tuple  # ggml order: (ne0 = row length, ne1, ne2)
    kind: str  # "quant" | "normal" | "uniform"
    scale: float  # d_sigma for quant, sigma for normal, (lo, hi) midpoint spread for uniform
    lo: float = 0.0
    hi: float = 0.0

    @property
    def nbytes(self) -> int:
        rows = int(np.prod(self.shape[1:])) if len(self.shape) > 1 else 1
        return row_bytes(self.qtype, self.shape[0]) * rows


def tensor_bytes(spec: TensorSpec, seed: int, index: int) -> Iterable[np.ndarray]:
    """Yields the tensor's bytes in chunks (deterministic in (seed, index))."""
    if spec.qtype in (F32, F16):
        n = int(np.prod(spec.shape))
        rng = _rng(seed, index, 0)
        if spec.kind == "normal":
            v = rng.normal(0.0, spec.scale, n)
        else:
            v = rng.uniform(spec.lo, spec.hi, n)
        yield (v.astype(np.float32) if spec.qtype == F32 else v.astype(np.float16)).view(np.uint8)
        return
    blck, nb = BLOCK[spec.qtype]
    total = spec.nbytes // nb
    for c, b0 in enumerate(range(0, total, CHUNK_BLOCKS)):
        n = min(CHUNK_BLOCKS, total - b0)
        yield quant_blocks(spec.qtype, n, _rng(seed, index, c), spec.scale).reshape(-1)


def tensor_array(spec: TensorSpec, seed: int, index: int) -> np.ndarray:
    return np.concatenate(list(tensor_bytes(spec, seed, index)))


# ------------------------------------------------------------------------------------------------
# qwen3moe model description
# ------------------------------------------------------------------------------------------------
@dataclasses.dataclass
class ModelConfig:
    name: str
    n_layer: int
    D: int
    n_head: int
    n_kv: int
    hd: int
    n_expert: int
    n_used: int
    FF: int
    n_vocab: int
    ctx_train: int = 4096
    rope_base: float = 1e6
    eps: float = 1e-6
    embd_type: int = Q4_K
    attn_types: tuple = (Q4_K, Q4_K, Q4_K, Q4_K)  # q, k, v, o
    expert_types: tuple = (Q4_K, Q4_K, Q6_K)  # gate, up, down
    output_type: int = Q6_K
    # scale parameters: per-type d sigma for quantized tensors, sigma for F32 tensors
    d_sigma: dict = dataclasses.field(default_factory=dict)
    f32_sigma: float = 0.02
    norm_kind: str = "uniform"  # norm weights: "uniform" (0.8..1.2) or "normal" (N(0, f32_sigma))
    seed: int = 0

    def tensors(self) -> list:
        QD, KD = self.n_head * self.hd, self.n_kv * self.hd
        ds = lambda t, default: self.d_sigma.get(t, default)  # noqa: E731

        def qspec(name, qt, shape):
            if qt in (F32, F16):
                return TensorSpec(name, qt, shape, "normal", self.f32_sigma)
            return TensorSpec(name, qt, shape, "quant", ds(name.split(".")[-2], ds(qt, 0.01)))

        def norm(name, n):
            if self.norm_kind == "normal":
                return TensorSpec(name, F32, (n,), "normal", self.f32_sigma)
            return TensorSpec(name, F32, (n,), "uniform", 0.0, 0.8, 1.2)

        out = [qspec("token_embd.weight", self.embd_type, (self.D, self.n_vocab)),
               qspec("output.weight", self.output_type, (self.D, self.n_vocab)),
               norm("output_norm.weight", self.D)]
        tq, tk, tv, to = self.attn_types
        tg, tu, td = self.expert_types
        for l in range(self.n_layer):
            p = f"blk.{l}."
            out += [norm(p + "attn_norm.weight", self.D), norm(p + "ffn_norm.weight", self.D),
                    norm(p + "attn_q_norm.weight", self.hd), norm(p + "attn_k_norm.weight", self.hd),
                    qspec(p + "attn_q.weight", tq, (self.D, QD)), qspec(p + "attn_k.weight", tk, (self.D, KD)),
                    qspec(p + "attn_v.weight", tv, (self.D, KD)), qspec(p + "attn_output.weight", to, (QD, self.D)),
                    TensorSpec(p + "ffn_gate_inp.weight", F32, (self.D, self.n_expert), "normal", self.f32_sigma),
                    qspec(p + "ffn_gate_exps.weight", tg, (self.D, self.FF, self.n_expert)),
                    qspec(p + "ffn_up_exps.weight", tu, (self.D, self.FF, self.n_expert)),
                    qspec(p + "ffn_down_exps.weight", td, (self.FF, self.D, self.n_expert))]
        return out

    def metadata(self) -> list:
        a = "qwen3moe."
        u32 = [("block_count", self.n_layer), ("context_length", self.ctx_train), ("embedding_length", self.D),
               ("attention.head_count", self.n_head), ("attention.head_count_kv", self.n_kv),
               ("attention.key_length", self.hd), ("attention.value_length", self.hd),
               ("expert_count", self.n_expert), ("expert_used_count", self.n_used),
               ("expert_feed_forward_length", self.FF)]
        kv = [("general.architecture", "str", "qwen3moe"), ("general.alignment", "u32", 32)]
        kv += [(a + k, "u32", v) for k, v in u32]
        kv += [(a + "rope.freq_base", "f32", self.rope_base), (a + "attention.layer_norm_rms_epsilon", "f32", self.eps)]
        # byte-level BPE table: 256 byte tokens, merges to fill the vocabulary, 3 specials
        toks = byte_tokens()
        merges = []
        n_merge = max(0, self.n_vocab - 256 - 3)
        for i in range(n_merge):
            a0, b0 = toks[97 + (i % 26)], toks[97 + ((i // 26) % 26)]
            toks.append(f"{a0}{b0}#{i}" if i >= 26 * 26 else a0 + b0)
            merges.append(f"{a0} {b0}")
        toks += ["<|im_start|>", "<|im_end|>", "<|endoftext|>"]
        kv += [("tokenizer.ggml.model", "str", "gpt2"), ("tokenizer.ggml.pre", "str", "qwen2"),
               ("tokenizer.ggml.tokens", "arr_str", toks[:self.n_vocab]),
               ("tokenizer.ggml.merges", "arr_str", merges[:1024]),
               ("tokenizer.ggml.eos_token_id", "u32", self.n_vocab - 2)]
        return kv


def byte_tokens() -> list:
    """GPT-2 byte-to-unicode mapping, one token per byte value."""
    bs = list(range(33, 127)) + list(range(161, 173)) + list(range(174, 256))
    cs = bs[:]
    n = 0
    for b in range(256):
        if b not in bs:
            bs.append(b)
            cs.append(256 + n)
            n += 1
    m = dict(zip(bs, cs))
    return [chr(m[b]) for b in range(256)]


# Configurations (BASELINE.json "configs").
def config1_tiny(seed: int = 1) -> ModelConfig:
    """Config 1: 2 layers, D 256, 4q/2kv heads of 64, 8 experts top-2, FF 256, vocab 512.
    Attention/router/norm/embedding F32 ~N(0, 0.02); experts all Q4_K with d, dmin ~|N(0, 0.01)|;
    output Q6_K (d ~|N(0, 0.01)|)."""
    return ModelConfig("tiny-q4k", n_layer=2, D=256, n_head=4, n_kv=2, hd=64, n_expert=8, n_used=2, FF=256,
                       n_vocab=512, ctx_train=512, rope_base=1e4, embd_type=F32, attn_types=(F32, F32, F32, F32),
                       expert_types=(Q4_K, Q4_K, Q4_K), output_type=Q6_K, norm_kind="normal", seed=seed)


# Unit-gain d sigmas for deep random models: a Q4_K weight d*s*q - dmin*m has a standard deviation of
# about 150*d for uniform scales/nibbles and a Q6_K weight d*sc*q about 340*d, so d = 1/(150*sqrt(K))
# (resp. 1/(340*sqrt(K))) keeps each projection near unit gain and the 48-layer residual stream finite.
def _unit_d(qtype: int, k: int) -> float:
    return 1.0 / ({Q4_K: 150.0, Q5_K: 300.0, Q6_K: 340.0, Q8_0: 75.0}[qtype] * np.sqrt(k))


def config4_30b(n_layer: int = 48, seed: int = 4) -> ModelConfig:
    """Config 4: Qwen3-30B-A3B shape, Q4_K attention/gate/up/embedding, Q6_K down/output."""
    D, QD, FF = 2048, 32 * 128, 768
    d = {"attn_q": _unit_d(Q4_K, D), "attn_k": _unit_d(Q4_K, D), "attn_v": _unit_d(Q4_K, D),
         "attn_output": _unit_d(Q4_K, QD), "ffn_gate_exps": _unit_d(Q4_K, D), "ffn_up_exps": _unit_d(Q4_K, D),
         "ffn_down_exps": _unit_d(Q6_K, FF), "output": _unit_d(Q6_K, D), "token_embd": 1.0 / 150.0}
    return ModelConfig("qwen3-30b-a3b-shape", n_layer=n_layer, D=D, n_head=32, n_kv=4, hd=128, n_expert=128,
                       n_used=8, FF=FF, n_vocab=151936, ctx_train=40960, rope_base=1e6, embd_type=Q4_K,
                       attn_types=(Q4_K, Q4_K, Q4_K, Q4_K), expert_types=(Q4_K, Q4_K, Q6_K), output_type=Q6_K,
                       d_sigma=d, f32_sigma=0.02, seed=seed)


def config_kquant_small(n_layer: int = 3, seed: int = 6) -> ModelConfig:
    """A small model with the config-4 structure (every projection K-quant, so the engine takes its
    tensor-core GEMV/GEMM paths): D 512, 8q/2kv heads of 64, 16 experts top-4, FF 256, vocab 1024;
    Q4_K q/k/v/embedding/gate, Q5_K attention output and up, Q6_K down and output."""
    D, QD, FF = 512, 8 * 64, 256
    d = {"attn_q": _unit_d(Q4_K, D), "attn_k": _unit_d(Q4_K, D), "attn_v": _unit_d(Q4_K, D),
         "attn_output": _unit_d(Q5_K, QD), "ffn_gate_exps": _unit_d(Q4_K, D), "ffn_up_exps": _unit_d(Q5_K, D),
         "ffn_down_exps": _unit_d(Q6_K, FF), "output": _unit_d(Q6_K, D), "token_embd": 1.0 / 150.0}
    return ModelConfig("kquant-small", n_layer=n_layer, D=D, n_head=8, n_kv=2, hd=64, n_expert=16, n_used=4, FF=FF,
                       n_vocab=1024, ctx_train=512, rope_base=1e6, embd_type=Q4_K,
                       attn_types=(Q4_K, Q4_K, Q4_K, Q5_K), expert_types=(Q4_K, Q5_K, Q6_K), output_type=Q6_K,
                       d_sigma=d, f32_sigma=0.02, seed=seed)


def config5_235b(n_layer: int = 94, seed: int = 5) -> ModelConfig:
    """Config 5: Qwen3-235B-A22B shape (EP workload), Q4_K attention/gate/up, Q6_K down/output."""
    D, QD, FF = 4096, 64 * 128, 1536
    d = {"attn_q": _unit_d(Q4_K, D), "attn_k": _unit_d(Q4_K, D), "attn_v": _unit_d(Q4_K, D),
         "attn_output": _unit_d(Q4_K, QD), "ffn_gate_exps": _unit_d(Q4_K, D), "ffn_up_exps": _unit_d(Q4_K, D),
         "ffn_down_exps": _unit_d(Q6_K, FF), "output": _unit_d(Q6_K, D), "token_embd": 1.0 / 150.0}
    return ModelConfig("qwen3-235b-a22b-shape", n_layer=n_layer, D=D, n_head=64, n_kv=4, hd=128, n_expert=128,
                       n_used=8, FF=FF, n_vocab=151936, ctx_train=40960, rope_base=1e6, embd_type=Q4_K,
                       d_sigma=d, f32_sigma=0.02, seed=seed)


# ------------------------------------------------------------------------------------------------
# GGUF v3 writer (streaming; layout as parsed by GGUF::load, qwen3moe.cpp:285-347)
# ------------------------------------------------------------------------------------------------
def _gguf_str(s: str) -> bytes:
    b = s.encode("utf-8")
    return struct.pack("<Q", len(b)) + b


def _gguf_kv(key: str, kind: str, val) -> bytes:
    out = _gguf_str(key)
    if kind == "str":
        return out + struct.pack("<I", 8) + _gguf_str(val)
    if kind == "u32":
        return out + struct.pack("<II", 4, val)
    if kind == "f32":
        return out + struct.pack("<If", 6, val)
    if kind == "arr_str":
        return out + struct.pack("<IIQ", 9, 8, len(val)) + b"".join(_gguf_str(s) for s in val)
    raise ValueError(kind)


def _layout(cfg: ModelConfig):
    """(header bytes, tensor specs, data offsets, total file size) of ``cfg``'s GGUF v3 file."""
    specs = cfg.tensors()
    align = 32
    header = bytearray(b"GGUF" + struct.pack("<IQQ", 3, len(specs), len(cfg.metadata())))
    for k, kind, v in cfg.metadata():
        header += _gguf_kv(k, kind, v)
    offsets, off = [], 0
    for s in specs:
        offsets.append(off)
        off += (s.nbytes + align - 1) // align * align
    for s, o in zip(specs, offsets):
        header += _gguf_str(s.name) + struct.pack("<I", len(s.shape))
        header += b"".join(struct.pack("<Q", n) for n in s.shape) + struct.pack("<IQ", s.qtype, o)
    header += b"\0" * ((-len(header)) % align)
    return bytes(header), specs, offsets, len(header) + off


def _write_chunks(args):
    """Pool worker: writes chunks [c0, c1) of tensor ``spec`` (index i of its model) at their offsets."""
    path, spec, i, c0, c1, base, seed = args
    fd = os.open(path, os.O_WRONLY)
    try:
        blck, nb = BLOCK[spec.qtype]
        total = spec.nbytes // nb
        for c in range(c0, c1):
            b0 = c * CHUNK_BLOCKS
            n = min(CHUNK_BLOCKS, total - b0)
            data = quant_blocks(spec.qtype, n, _rng(seed, i, c), spec.scale).reshape(-1)
            os.pwrite(fd, data.tobytes(), base + b0 * nb)
    finally:
        os.close(fd)
    return c1 - c0


def write_gguf(path: str, cfg: ModelConfig, progress: Callable[[str], None] | None = None, workers: int = 0) -> str:
    """Writes ``cfg`` as a GGUF v3 file at ``path`` (atomically). Returns the path.

    workers > 0 generates the quantized tensors' chunks in that many spawned processes (same bytes:
    every chunk's generator is keyed by (seed, tensor index, chunk index)). Call it before any CUDA
    work in the calling process."""
    header, specs, offsets, size = _layout(cfg)
    tmp = path + ".tmp"
    if workers <= 0:
        with open(tmp, "wb") as f:
            f.write(header)
            for i, (s, o) in enumerate(zip(specs, offsets)):
                if progress and i % 12 == 0:
                    progress(f"{s.name} ({i + 1}/{len(specs)})")
                n = 0
                for chunk in tensor_bytes(s, cfg.seed, i):
                    f.write(chunk.tobytes())
                    n += chunk.size
                assert n == s.nbytes, (s.name, n, s.nbytes)
                f.write(b"\0" * ((-n) % 32))
        os.replace(tmp, path)
        return path
    import multiprocessing as mp
    with open(tmp, "wb") as f:
        f.write(header)
        f.truncate(size)  # padding and alignment gaps read as zeros
        for i, (s, o) in enumerate(zip(specs, offsets)):
            if s.qtype in (F32, F16):
                f.seek(len(header) + o)
                for chunk in tensor_bytes(s, cfg.seed, i):
                    f.write(chunk.tobytes())
    jobs = []
    for i, (s, o) in enumerate(zip(specs, offsets)):
        if s.qtype in (F32, F16):
            continue
        nchunk = -(-(s.nbytes // BLOCK[s.qtype][1]) // CHUNK_BLOCKS)
        for c in range(nchunk):
            jobs.append((tmp, s, i, c, c + 1, len(header) + o, cfg.seed))
    done = 0
    with mp.get_context("spawn").Pool(workers) as pool:
        for n in pool.imap_unordered(_write_chunks, jobs, chunksize=1):
            done += n
            if progress and done % 64 == 0:
                progress(f"{done}/{len(jobs)} chunks")
    os.replace(tmp, path)
    return path


def config_digest(cfg: ModelConfig) -> str:
    return hashlib.sha256(repr(dataclasses.asdict(cfg)).encode()).hexdigest()[:16]


def cached_gguf(cfg: ModelConfig, directory: str | None = None, progress=None, workers: int = 0) -> str:
    """Path of ``cfg``'s GGUF under ``directory`` (default $EAHMMF_MODEL_DIR or /tmp/eahmmf_models),
    generating it when absent."""
    directory = directory or os.environ.get("EAHMMF_MODEL_DIR", "/tmp/eahmmf_models")
    os.makedirs(directory, exist_ok=True)
    path = os.path.join(directory, f"{cfg.name}-L{cfg.n_layer}-{config_digest(cfg)}.gguf")
    if not os.path.exists(path):
        write_gguf(path, cfg, progress, workers)
    return path


# ------------------------------------------------------------------------------------------------
# Config 2/3 expert sets (no GGUF needed): per-expert gate/up/down byte arrays
# ------------------------------------------------------------------------------------------------
@dataclasses.dataclass
class ExpertSet:
    D: int
    FF: int
    n_expert: int
    types: tuple  # gate, up, down
    gate: np.ndarray  # (E, FF * row_bytes(gate)) uint8
    up: np.ndarray
    down: np.ndarray

    @property
    def row_bytes(self) -> tuple:
        tg, tu, td = self.types
        return row_bytes(tg, self.D), row_bytes(tu, self.D), row_bytes(td, self.FF)

    @property
    def expert_bytes(self) -> int:
        return self.gate.shape[1] + self.up.shape[1] + self.down.shape[1]


def expert_set(D: int = 2048, FF: int = 768, n_expert: int = 128, types=(Q4_K, Q4_K, Q6_K), seed: int = 2,
               d_sigma: float = 0.01, experts: range | None = None) -> ExpertSet:
    """Config 2/3 experts: gate/up [FF x D], down [D x FF], d ~|N(0, d_sigma)| per block. `experts`
    (optional) generates only that range of the set's experts (an expert-parallel rank's shard): each
    expert's bytes come from its own seed, so a shard equals the same slice of the whole set."""
    tg, tu, td = types
    ids = range(n_expert) if experts is None else experts
    comps = []
    for c, (qt, rows, k) in enumerate(((tg, FF, D), (tu, FF, D), (td, D, FF))):
        blck, nb = BLOCK[qt]
        nblk = rows * (k // blck)
        arr = np.empty((len(ids), nblk * nb), np.uint8)
        for i, e in enumerate(ids):
            arr[i] = quant_blocks(qt, nblk, _rng(seed, c, e), d_sigma).reshape(-1)
        comps.append(arr)
    return ExpertSet(D, FF, len(ids), tuple(types), *comps)


def activations(T: int, D: int, seed: int) -> np.ndarray:
    return _rng(seed, 0xA11).normal(0.0, 1.0, (T, D)).astype(np.float32)


def router_logits(T: int, E: int, seed: int, zipf_bias: float = 0.0) -> np.ndarray:
    """Router logits ~N(0, 1), optionally plus a log-Zipf(s) popularity bias per expert (config 3)."""
    rng = _rng(seed, 0x1061)
    lg = rng.normal(0.0, 1.0, (T, E))
    if zipf_bias:
        rank = rng.permutation(E) + 1
        lg = lg - zipf_bias * np.log(rank)[None, :]
    return lg.astype(np.float32)


def ragged_batch(n_seq: int = 64, lo: int = 1, hi: int = 512, seed: int = 3) -> np.ndarray:
    """Config 3: per-sequence token counts uniform in [lo, hi]."""
    return _rng(seed, 0x5E9).integers(lo, hi + 1, size=n_seq)
