"""Write the golden fixtures of tests/golden/ from the reference itself (run where the reference tree exists).

    python tests/golden/make_golden.py REFERENCE_ROOT      (or IMI_REFERENCE=REFERENCE_ROOT in the environment)

For the seeded synthetic models of nunchi_b200.synth it records:
  * ref_<model>.npz   - outputs of the reference's own imi_seoul (imi/core/seoul.cpp + tables.cpp, built unmodified
                        into oracle/_ref): per-position hidden and logits of a greedy-free token sequence (step), the
                        per-position hidden of step_batch over input vectors, and 8-bit cuts / 4-bit table outputs of
                        the reference's table kernels (imi_q8::from, imi_q4_group, imi_q4_group2, imi_q4_group_batch);
  * truth_<model>.npz - the fp64 truth key of the same token sequence, from the reference's imi/ref/ref_exact.py run
                        unmodified on the same file (hidden and logits rounded to fp32 by that script).
Large outputs are summarised (first positions in full, then top-k ids/values and float sums) so the fixtures stay small.
"""
from __future__ import annotations

import hashlib
import os
import struct
import subprocess
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)
HERE = os.path.dirname(os.path.abspath(__file__))

import oracle  # noqa: E402
from nunchi_b200 import synth  # noqa: E402

# model -> (token positions stepped, positions of the reference's logits kept in full, positions of the truth key's
# logits kept in full, embedding positions for step_batch). The Seoul truth key keeps all 32 positions in full (the
# max-abs error budget needs whole score vectors); imi's own error there is measured live with the oracle, which is
# pinned bit for bit to the reference.
PLAN = {"tiny": (32, 32, 32, 20), "wide_heads": (32, 32, 32, 12), "seoul": (32, 2, 32, 4)}


def write_answer_key(path, toks, hid, lg):
    """imi's REF.bin layout (imi/ref/ref_llama.cpp:5): int32 n_embd, n_vocab, n; per position int32 token, f32 hidden,
    f32 logits. ref_exact.py reads the token list from it."""
    with open(path, "wb") as f:
        f.write(struct.pack("3i", hid.shape[1], lg.shape[1], len(toks)))
        for i, t in enumerate(toks):
            f.write(struct.pack("i", int(t)))
            f.write(hid[i].astype(np.float32).tobytes())
            f.write(lg[i].astype(np.float32).tobytes())


def read_answer_key(path):
    with open(path, "rb") as f:
        ne, nv, n = struct.unpack("3i", f.read(12))
        H, L = [], []
        for _ in range(n):
            f.read(4)
            H.append(np.frombuffer(f.read(4 * ne), np.float32))
            L.append(np.frombuffer(f.read(4 * nv), np.float32))
    return np.array(H), np.array(L)


def summarise(prefix, lg, full, out):
    """first `full` positions of the logits in full; for every position the top-16 and float64 sums."""
    out[prefix + "_full"] = lg[:full]
    top = np.argsort(-lg, axis=1, kind="stable")[:, :16]
    out[prefix + "_top_ids"] = top.astype(np.int32)
    out[prefix + "_top_vals"] = np.take_along_axis(lg, top, 1)
    out[prefix + "_sum"] = lg.astype(np.float64).sum(1)
    out[prefix + "_sumsq"] = (lg.astype(np.float64) ** 2).sum(1)
    out[prefix + "_sha256"] = np.array([hashlib.sha256(r.tobytes()).hexdigest() for r in lg])


def main(ref_root):
    for name, (n, full, full_truth, n_emb) in PLAN.items():
        path = synth.cached_gguf(name, 0)
        r = oracle.Reference(path, n_ctx=256)
        toks = synth.random_ids(n, r.n_vocab, 7)
        H, L = [], []
        for t in toks:
            r.step(int(t))
            H.append(r.hidden)
            L.append(r.logits)
        H, L = np.array(H), np.array(L)
        out = {"tokens": toks, "hidden": H}
        summarise("logits", L, full, out)
        # step_batch over input vectors (the ears' hand-off, config 3 in miniature): N(0,1) * 0.5, seed 3
        emb = (0.5 * np.random.default_rng(3).standard_normal((n_emb, r.n_embd))).astype(np.float32)
        r.reset()
        out["batch_embd"] = emb
        out["batch_hidden"] = r.step_batch(embd=emb, want_logits=True, hidden_all=True)
        bl = r.logits[None]
        summarise("batch_logits", bl, 1, out)
        # kernel level: the reference's own cut and 4-bit kernels on a seeded table
        rng = np.random.default_rng(11)
        rows, cols = 64, 512
        q4 = synth._q4_0(rng, rows, cols).reshape(-1)
        x = rng.standard_normal((5, cols)).astype(np.float32)
        x[0, :32] = 0.0
        out["kat_q4"], out["kat_x"] = q4, x
        cq = [oracle.ref_cut(v) for v in x]
        out["kat_q"] = np.stack([c[0] for c in cq])
        out["kat_d"] = np.stack([c[1] for c in cq])
        out["kat_s"] = np.stack([c[2] for c in cq])
        out["kat_out1"] = oracle.ref_q4_matvec(q4, rows, cols, x[:1])
        out["kat_out2"] = oracle.ref_q4_matvec(q4, rows, cols, x[:2])
        out["kat_out5"] = oracle.ref_q4_matvec(q4, rows, cols, x)
        np.savez_compressed(os.path.join(HERE, f"ref_{name}.npz"), **out)
        del r
        # fp64 truth key of the same tokens (the reference's own script, unmodified)
        key = f"/tmp/imi_golden_{name}_ref.bin"
        write_answer_key(key, toks, H, L)
        import gguf
        gdir = os.path.dirname(os.path.dirname(gguf.__file__))
        tkey = f"/tmp/imi_golden_{name}_truth.bin"
        subprocess.run([sys.executable, os.path.join(ref_root, "imi", "ref", "ref_exact.py"), gdir, path, key,
                        str(len(toks)), tkey], check=True, capture_output=True)
        th, tl = read_answer_key(tkey)
        tout = {"tokens": toks, "hidden": th}
        summarise("logits", tl, full_truth, tout)
        np.savez_compressed(os.path.join(HERE, f"truth_{name}.npz"), **tout)
        print(name, "written", flush=True)


if __name__ == "__main__":
    root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("IMI_REFERENCE")
    if not root:
        sys.exit("usage: make_golden.py REFERENCE_ROOT (or set IMI_REFERENCE)")
    main(root)
