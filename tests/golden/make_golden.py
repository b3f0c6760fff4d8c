"""Generate the golden fixtures in this directory from the REFERENCE itself.

Runs the unmodified reference CPU ops (oracle/_ref/libgenllm_ref.so and
libgenllm_ref_ops.so, compiled from the Genllm sources by oracle/Makefile) on
the seeded cases of cases.py and stores their outputs. Needs the reference tree (only present where the
fixtures are made); the tests only read the .npz files.

    make -C oracle && python tests/golden/make_golden.py
"""
import hashlib
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
sys.path.insert(0, HERE)

from cases import CONFIG1, FLASH, KV_FORMAT, QK_ROPE, SMALL  # noqa: E402
from genllm_b200.synth import fragmented_case, heads_major, qk_rope_case  # noqa: E402
from oracle.oracle import RefOps, RefSession, ref_flash_attention, run_ref_case  # noqa: E402


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def main():
    for name, kw, causal in SMALL:
        c = fragmented_case(**kw)
        out, kp, vp, k_ids, v_ids, nc = run_ref_case(c, causal)
        np.savez_compressed(os.path.join(HERE, f"{name}.npz"), q=c.q, k_new=c.k_new, v_new=c.v_new,
                            k_pool=c.k_pool, v_pool=c.v_pool, k_ids_in=c.k_ids, v_ids_in=c.v_ids,
                            k_free_order=c.k_free_order, v_free_order=c.v_free_order,
                            out_bf16=out, k_pool_after=kp, v_pool_after=vp, k_ids=k_ids, v_ids=v_ids,
                            num_cached=nc)
        print(name, out.shape, nc)
    name, kw, causal = CONFIG1
    c = fragmented_case(**kw)
    out, kp, vp, k_ids, v_ids, nc = run_ref_case(c, causal)
    np.savez_compressed(os.path.join(HERE, f"{name}.npz"), out_bf16=out, k_ids=k_ids, v_ids=v_ids,
                        num_cached=nc, inputs_sha=np.array([sha(c.k_pool), sha(c.v_pool), sha(c.q),
                                                            sha(c.k_new), sha(c.v_new)]),
                        pools_after_sha=np.array([sha(kp), sha(vp)]))
    print(name, out.shape, nc)
    make_qk_rope()
    make_flash()
    make_kv_format()


def flash_inputs(seed, B, Hq, Hkv, S):
    from genllm_b200.synth import randn_bf16
    rng = np.random.default_rng(seed)
    return (randn_bf16(rng, (B, Hq, S, 128)), randn_bf16(rng, (B, Hkv, S, 128)), randn_bf16(rng, (B, Hkv, S, 128)))


def make_flash():
    """FlashAttentionImpl<CPU> (src/backend/cpu/attention.cpp:39-120)."""
    for name, seed, B, Hq, Hkv, S, causal in FLASH:
        q, k, v = flash_inputs(seed, B, Hq, Hkv, S)
        out = ref_flash_attention(q, k, v, float(1 / np.sqrt(128)), causal)
        np.savez_compressed(os.path.join(HERE, f"{name}.npz"), out_bf16=out,
                            inputs_sha=np.array([sha(q), sha(k), sha(v)]))
        print(name, out.shape)


def make_qk_rope():
    """Reference pipeline of src/model/Qwen3.cpp:136-154: reshape_permute to
    [H][S][D], per-head rms_norm, apply_rope at start_pos."""
    R = RefOps()
    for name, kw, max_seq in QK_ROPE:
        c = qk_rope_case(**kw)
        cos, sin = R.rope_cache(c.theta, c.head_dim, max_seq)
        q4 = heads_major(c.q_flat, c.n_q_heads)
        k4 = heads_major(c.k_flat, c.n_kv_heads)
        qn = R.rms_norm_bf16(q4, c.q_norm_w, c.eps)
        kn = R.rms_norm_bf16(k4, c.k_norm_w, c.eps)
        qr = R.apply_rope_bf16(qn, cos, sin, c.start_pos)
        kr = R.apply_rope_bf16(kn, cos, sin, c.start_pos)
        np.savez_compressed(os.path.join(HERE, f"{name}.npz"), q_rope=qr, k_rope=kr, q_normed=qn, k_normed=kn,
                            cache_sha=np.array([sha(cos), sha(sin)]),
                            inputs_sha=np.array([sha(c.q_flat), sha(c.k_flat), sha(c.q_norm_w), sha(c.k_norm_w)]))
        print(name, qr.shape, kr.shape)


def fp8_export_numpy(x_bits: np.ndarray):
    """Expected e4m3 export of [H][n][D] bf16 bits, independent of the C
    oracle: numpy fp32 block amax / scale / product, torch's float8_e4m3fn
    conversion (round to nearest even) after clamping to +-448, NaN -> 0x7F."""
    import torch
    H, n, D = x_bits.shape
    nb = (n + 15) // 16
    x = (x_bits.astype(np.uint32) << 16).view(np.float32)
    q = np.zeros(x.shape, np.uint8)
    scales = np.zeros((H, nb), np.float32)
    for h in range(H):
        for b in range(nb):
            blk = x[h, 16 * b:16 * b + 16]
            a = np.abs(blk[np.isfinite(blk)])
            amax = np.float32(a.max()) if a.size else np.float32(0)
            with np.errstate(divide="ignore", over="ignore"):
                inv = np.float32(448) / amax
            scale = amax / np.float32(448) if np.isfinite(inv) else np.float32(1)
            inv = inv if np.isfinite(inv) else np.float32(1)
            y = np.clip(blk * inv, np.float32(-448), np.float32(448)).astype(np.float32)
            e = torch.from_numpy(np.ascontiguousarray(y)).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
            q[h, 16 * b:16 * b + 16] = np.where(np.isnan(y), np.uint8(0x7F), e)
            scales[h, b] = scale
    return q, scales


def make_kv_format():
    """Pages from the reference's append_kv_from_tensor
    (src/core/page_attention.cpp:104-139), called once per chunk."""
    from genllm_b200.synth import kv_format_values
    for name, seed, hkv, chunks, pages in KV_FORMAT:
        n = sum(chunks)
        K, V = kv_format_values(seed, hkv, n)
        R = RefSession(1, hkv, 128, pages)
        p0 = 0
        for c in chunks:
            R.append_kv(0, np.ascontiguousarray(K[:, p0:p0 + c]), np.ascontiguousarray(V[:, p0:p0 + c]), c)
            p0 += c
        k_ids, v_ids, nc = R.table(0)
        kq, ks = fp8_export_numpy(K)
        vq, vs = fp8_export_numpy(V)
        # K and V themselves are regenerated from the seed (checksums here).
        np.savez_compressed(os.path.join(HERE, f"{name}.npz"), k_pool=R.pool_view(0, 0).copy(),
                            v_pool=R.pool_view(0, 1).copy(), k_ids=k_ids, v_ids=v_ids, num_cached=nc,
                            kv_sha=np.array([sha(K), sha(V)]), k_fp8=kq, v_fp8=vq, k_scales=ks, v_scales=vs)
        R.close()
        print(name, K.shape, nc, len(k_ids))


if __name__ == "__main__":
    main()
