"""Seeded synthetic Seoul-shaped GGUF files (LFM3 hybrid backbone, Q4_0 tables, tied Q4_0 word table).

The engine loads weights from GGUF exactly as imi does (imi/core/seoul.cpp:93-186 reads the `lfm3.*` keys and the
`blk.N.*` tensor names below). No real checkpoint is available offline, so benchmarks and tests use random-init
weights drawn here from a fixed seed:

* Q4_0 tables: 4-bit codes uniform in 0..15, fp16 block scales U(0.002, 0.01), 32-wide blocks;
* short-conv taps fp32 N(0, 0.1) (file layout [channel][tap], kernel 3 -> `lfm3.shortconv.l_cache` = 3);
* RMSNorm weights fp32 1 + 0.1 N(0, 1) (q/k norms included, imi requires them: seoul.cpp:149-150);
* tied embedding / LM head `token_embd.weight` in Q4_0.

The GGUF container is written by this module directly (format version 3: header, key/values, tensor infos,
32-byte aligned data), so nothing outside numpy is needed on the GPU box.
"""
from __future__ import annotations

import os
import struct
from dataclasses import dataclass, replace, field

import numpy as np

# ggml type ids used here
GGML_F32, GGML_F16, GGML_Q4_0, GGML_Q4_1, GGML_Q6_K = 0, 1, 2, 3, 14
# gguf value types
_U32, _I32, _F32, _BOOL, _STR, _ARR, _U64 = 4, 5, 6, 7, 8, 9, 10
ALIGN = 32


@dataclass(frozen=True)
class Shape:
    n_embd: int = 2048
    n_layer: int = 16
    attn_layers: tuple = (2, 5, 8, 10, 12, 14)   # LFM2-1.2B's attention placement
    n_head: int = 32
    n_head_kv: int = 8
    head_dim: int = 64
    n_ff: int = 8192
    l_cache: int = 3                              # conv kernel width; d_conv = l_cache - 1
    n_vocab: int = 97496
    rope_base: float = 1e6
    eps: float = 1e-5
    n_swa: int = 0                                # sliding window (0 = none)
    swa_layers: tuple = ()                        # attention layers that use the window
    rope_freqs: bool = False                      # write a rope_freqs.weight table
    word_q6k: bool = False                        # the word table in Q6_K (the product's own format) instead of Q4_0
    tables_q41: bool = False                      # the layer tables in Q4_1 (d and m per block) instead of Q4_0

    @property
    def kvd(self) -> int:
        return self.n_head_kv * self.head_dim

    def is_attn(self, il: int) -> bool:
        return il in self.attn_layers


SEOUL = Shape()
# small shapes for the CPU suite and quick GPU parity checks. n_embd must be a multiple of 256 (imi reads the word
# table in 256-wide pieces, seoul.cpp:236,363) and n_head a multiple of 8 (the stacked q|k|v|gate table is read in
# 8-row groups, tables.cpp:68). n_head * head_dim equals n_embd, as in Seoul: the reference's batched read cuts the
# attention output with the n_embd-wide input shape (seoul.cpp:554,623), so only such shapes give it one meaning
TINY = Shape(n_embd=512, n_layer=4, attn_layers=(1, 3), n_head=8, n_head_kv=2, head_dim=64, n_ff=1024,
             n_vocab=1003)
SMALL = Shape(n_embd=512, n_layer=6, attn_layers=(2, 4), n_head=8, n_head_kv=2, head_dim=64, n_ff=1536,
              n_vocab=4099)
# the real Seoul geometry's attention (heads of 128, sliding-window layers, rope_freqs), scaled down
WIDE_HEADS = Shape(n_embd=1024, n_layer=4, attn_layers=(1, 2, 3), n_head=8, n_head_kv=2, head_dim=128, n_ff=2048,
                   n_vocab=2001, n_swa=8, swa_layers=(2,), rope_freqs=True)

# two query heads per kv head at head_dim 64, one attention layer with a window of 8 (the attention kernels' other
# group width and their windowed ring starts)
TINY_G2 = Shape(n_embd=512, n_layer=4, attn_layers=(1, 3), n_head=8, n_head_kv=4, head_dim=64, n_ff=1024,
                n_vocab=1003, n_swa=8, swa_layers=(3,))

# TINY with a Q6_K word table, as the product's own files have
TINY_Q6K = Shape(n_embd=512, n_layer=4, attn_layers=(1, 3), n_head=8, n_head_kv=2, head_dim=64, n_ff=1024,
                 n_vocab=1003, word_q6k=True)

# TINY with Q4_1 layer tables (a per-block minimum besides the scale)
TINY_Q41 = Shape(n_embd=512, n_layer=4, attn_layers=(1, 3), n_head=8, n_head_kv=2, head_dim=64, n_ff=1024,
                 n_vocab=1003, tables_q41=True)
# the Seoul shape with the product's own Q6_K word table
SEOUL_Q6K = replace(SEOUL, word_q6k=True)

SHAPES = {"seoul": SEOUL, "tiny": TINY, "small": SMALL, "wide_heads": WIDE_HEADS, "tiny_q6k": TINY_Q6K,
          "seoul_q6k": SEOUL_Q6K, "tiny_q41": TINY_Q41, "tiny_g2": TINY_G2}


def _q4_0(rng: np.random.Generator, rows: int, cols: int) -> np.ndarray:
    """A Q4_0 table [rows][cols/32 blocks] of 18-byte blocks: fp16 scale, 16 bytes of packed codes."""
    assert cols % 32 == 0
    nblk = rows * (cols // 32)
    out = np.empty((nblk, 18), np.uint8)
    out[:, :2] = rng.uniform(0.002, 0.01, nblk).astype(np.float16).view(np.uint8).reshape(nblk, 2)
    out[:, 2:] = rng.integers(0, 256, (nblk, 16), dtype=np.uint8)   # two uniform nibbles per byte
    return out


def _q6k(rng: np.random.Generator, rows: int, cols: int) -> np.ndarray:
    """A Q6_K table [rows][cols/256 blocks] of 210-byte blocks: ql[128], qh[64] (uniform 6-bit codes), int8 scales[16]
    in [-8, 8], fp16 d: values d * scale * (code - 32) of the Q4_0 tables' magnitude."""
    assert cols % 256 == 0
    nblk = rows * (cols // 256)
    out = np.empty((nblk, 210), np.uint8)
    out[:, :192] = rng.integers(0, 256, (nblk, 192), dtype=np.uint8)
    out[:, 192:208] = rng.integers(-8, 9, (nblk, 16)).astype(np.int8).view(np.uint8)
    out[:, 208:] = rng.uniform(2e-4, 6e-4, nblk).astype(np.float16).view(np.uint8).reshape(nblk, 2)
    return out


def _q4_1(rng: np.random.Generator, rows: int, cols: int) -> np.ndarray:
    """A Q4_1 table [rows][cols/32 blocks] of 20-byte blocks: fp16 d, fp16 m (about -8 d: values d*code + m centred),
    16 bytes of packed codes."""
    assert cols % 32 == 0
    nblk = rows * (cols // 32)
    out = np.empty((nblk, 20), np.uint8)
    d = rng.uniform(0.002, 0.01, nblk).astype(np.float32)
    out[:, :2] = d.astype(np.float16).view(np.uint8).reshape(nblk, 2)
    out[:, 2:4] = (-8.0 * d * rng.uniform(0.8, 1.2, nblk)).astype(np.float16).view(np.uint8).reshape(nblk, 2)
    out[:, 4:] = rng.integers(0, 256, (nblk, 16), dtype=np.uint8)
    return out


def _norm(rng, n):
    return (1.0 + 0.1 * rng.standard_normal(n)).astype(np.float32)


def tensors(shape: Shape, seed: int = 0):
    """Yield (name, ggml_type, ne (fastest first), bytes) in file order, drawing from one seeded generator."""
    rng = np.random.default_rng(seed)
    E, F = shape.n_embd, shape.n_ff
    QT, qt = (GGML_Q4_1, _q4_1) if shape.tables_q41 else (GGML_Q4_0, _q4_0)   # the layer tables' format
    if shape.word_q6k:
        yield "token_embd.weight", GGML_Q6_K, (E, shape.n_vocab), _q6k(rng, shape.n_vocab, E)
    else:
        yield "token_embd.weight", GGML_Q4_0, (E, shape.n_vocab), _q4_0(rng, shape.n_vocab, E)
    yield "output_norm.weight", GGML_F32, (E,), _norm(rng, E)
    if shape.rope_freqs:
        ff = (1.0 + rng.uniform(0.0, 3.0, shape.head_dim // 2)).astype(np.float32)
        yield "rope_freqs.weight", GGML_F32, (shape.head_dim // 2,), ff
    for il in range(shape.n_layer):
        p = f"blk.{il}."
        yield p + "attn_norm.weight", GGML_F32, (E,), _norm(rng, E)
        if shape.is_attn(il):
            H, D, kvd = shape.n_head, shape.head_dim, shape.kvd
            yield p + "attn_q.weight", QT, (E, H * D), qt(rng, H * D, E)
            yield p + "attn_k.weight", QT, (E, kvd), qt(rng, kvd, E)
            yield p + "attn_v.weight", QT, (E, kvd), qt(rng, kvd, E)
            yield p + "attn_gate.weight", QT, (E, H), qt(rng, H, E)
            yield p + "attn_output.weight", QT, (H * D, E), qt(rng, E, H * D)
            yield p + "attn_q_norm.weight", GGML_F32, (D,), _norm(rng, D)
            yield p + "attn_k_norm.weight", GGML_F32, (D,), _norm(rng, D)
        else:
            K = shape.l_cache
            taps = (0.1 * rng.standard_normal((E, K))).astype(np.float32)   # [channel][tap]
            yield p + "shortconv.conv.weight", GGML_F32, (K, E), taps
            yield p + "shortconv.in_proj.weight", QT, (E, 3 * E), qt(rng, 3 * E, E)
            yield p + "shortconv.out_proj.weight", QT, (E, E), qt(rng, E, E)
        yield p + "post_attention_norm.weight", GGML_F32, (E,), _norm(rng, E)
        yield p + "ffn_norm.weight", GGML_F32, (E,), _norm(rng, E)
        yield p + "ffn_gate.weight", QT, (E, F), qt(rng, F, E)
        yield p + "ffn_up.weight", QT, (E, F), qt(rng, F, E)
        yield p + "ffn_down.weight", QT, (F, E), qt(rng, E, F)
        yield p + "post_ffw_norm.weight", GGML_F32, (E,), _norm(rng, E)


def _s(x: str) -> bytes:
    b = x.encode()
    return struct.pack("<Q", len(b)) + b


def _kv(key: str, vtype: int, value) -> bytes:
    out = _s(key) + struct.pack("<I", vtype)
    if vtype == _U32:
        return out + struct.pack("<I", value)
    if vtype == _I32:
        return out + struct.pack("<i", value)
    if vtype == _F32:
        return out + struct.pack("<f", value)
    if vtype == _STR:
        return out + _s(value)
    if vtype == _ARR:
        et, vals = value
        body = struct.pack("<IQ", et, len(vals))
        if et == _BOOL:
            body += bytes(int(bool(v)) for v in vals)
        elif et == _F32:
            body += struct.pack(f"<{len(vals)}f", *vals)
        else:
            raise ValueError(et)
        return out + body
    raise ValueError(vtype)


def metadata(shape: Shape) -> list:
    kv = [
        ("general.architecture", _STR, "lfm3"),
        ("general.alignment", _U32, ALIGN),
        ("lfm3.block_count", _U32, shape.n_layer),
        ("lfm3.embedding_length", _U32, shape.n_embd),
        ("lfm3.feed_forward_length", _U32, shape.n_ff),
        ("lfm3.vocab_size", _U32, shape.n_vocab),
        ("lfm3.attention.head_count", _U32, shape.n_head),
        ("lfm3.attention.head_count_kv", _U32, shape.n_head_kv),
        ("lfm3.attention.key_length", _U32, shape.head_dim),
        ("lfm3.attention.value_length", _U32, shape.head_dim),
        ("lfm3.attention.layer_norm_rms_epsilon", _F32, shape.eps),
        ("lfm3.rope.freq_base", _F32, shape.rope_base),
        ("lfm3.rope.freq_base_swa", _F32, 1e4),
        ("lfm3.shortconv.l_cache", _U32, shape.l_cache),
        ("lfm3.attention.sliding_window", _U32, shape.n_swa),
        ("lfm3.attention.sliding_window_pattern", _ARR,
         (_BOOL, [il in shape.swa_layers for il in range(shape.n_layer)])),
    ]
    return kv


def write_gguf(path: str, shape: Shape = SEOUL, seed: int = 0, override: dict | None = None) -> str:
    """Write the seeded synthetic model to `path` (GGUF v3). Returns the path. `override` maps tensor names to
    (ggml type, ne, array) written in their place (files the engine must refuse, in the failure tests)."""
    ts = [(n, *override[n]) if override and n in override else (n, t, ne, d) for n, t, ne, d in tensors(shape, seed)]
    kv = metadata(shape)
    infos, off = [], 0
    for name, typ, ne, data in ts:
        infos.append(_s(name) + struct.pack("<I", len(ne)) + struct.pack(f"<{len(ne)}Q", *ne)
                     + struct.pack("<IQ", typ, off))
        off += (data.nbytes + ALIGN - 1) // ALIGN * ALIGN
    head = b"GGUF" + struct.pack("<IQQ", 3, len(ts), len(kv))
    head += b"".join(_kv(*e) for e in kv) + b"".join(infos)
    tmp = path + f".tmp{os.getpid()}"
    with open(tmp, "wb") as f:
        f.write(head)
        f.write(b"\0" * ((-len(head)) % ALIGN))
        for _, _, _, data in ts:
            f.write(np.ascontiguousarray(data).tobytes())
            f.write(b"\0" * ((-data.nbytes) % ALIGN))
    os.replace(tmp, path)
    return path


def cached_gguf(name: str = "seoul", seed: int = 0, directory: str | None = None) -> str:
    """Path of the synthetic model `name` for `seed`, writing it once per machine (under /dev/shm when present)."""
    shape = SHAPES[name]
    d = directory or os.environ.get("IMI_SYNTH_DIR") or ("/dev/shm" if os.path.isdir("/dev/shm") else "/tmp")
    path = os.path.join(d, f"imi_synth_{name}_s{seed}.gguf")
    if not os.path.exists(path):
        write_gguf(path, shape, seed)
    return path


def random_ids(n: int, n_vocab: int, seed: int) -> np.ndarray:
    """Uniform random token ids in [0, n_vocab) (the configs' prompts)."""
    return np.random.default_rng(seed).integers(0, n_vocab, n).astype(np.int32)


if __name__ == "__main__":
    import sys
    name = sys.argv[1] if len(sys.argv) > 1 else "seoul"
    print(cached_gguf(name, int(sys.argv[2]) if len(sys.argv) > 2 else 0))
