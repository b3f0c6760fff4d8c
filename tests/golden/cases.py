"""The golden cases: (name, fragmented_case kwargs, causal). Shared by the
fixture generator (make_golden.py) and the tests that read the fixtures."""

# Small cases store every input in the fixture; "config1" (Qwen3-0.6B layer,
# seed 0, 1024 prior tokens in 64 of 256 pages, append 1) stores only the
# outputs and checksums, its inputs being regenerated from the seed.
SMALL = [
    ("decode_g2_midpage", dict(seed=11, n_q_heads=4, n_kv_heads=2, head_dim=128, n_prior=37, pool_pages=8), True),
    ("decode_g2_newpage", dict(seed=12, n_q_heads=4, n_kv_heads=2, head_dim=128, n_prior=48, pool_pages=8), True),
    ("decode_g1", dict(seed=13, n_q_heads=2, n_kv_heads=2, head_dim=128, n_prior=21, pool_pages=6), True),
    ("decode_g4", dict(seed=14, n_q_heads=8, n_kv_heads=2, head_dim=128, n_prior=70, pool_pages=8), True),
    ("decode_g8", dict(seed=15, n_q_heads=8, n_kv_heads=1, head_dim=128, n_prior=33, pool_pages=6), True),
    ("decode_first_token", dict(seed=16, n_q_heads=4, n_kv_heads=2, head_dim=128, n_prior=0, pool_pages=4), True),
    ("chunk_causal", dict(seed=17, n_q_heads=4, n_kv_heads=2, head_dim=128, n_prior=10, pool_pages=8, n_new=29), True),
    ("chunk_noncausal", dict(seed=18, n_q_heads=4, n_kv_heads=2, head_dim=128, n_prior=10, pool_pages=8, n_new=29), False),
    ("chunk_from_empty", dict(seed=19, n_q_heads=4, n_kv_heads=2, head_dim=128, n_prior=0, pool_pages=8, n_new=40), True),
]

CONFIG1 = ("config1", dict(seed=0, n_q_heads=16, n_kv_heads=8, head_dim=128, n_prior=1024, pool_pages=256), True)

# QK-norm + RoPE (the step that produces the K the attention op appends):
# (name, qk_rope_case kwargs, max_seq of the RoPE table). The fixtures hold the
# reference's normalised + rotated Q and K ([H][S][D] bf16) and a checksum of
# its cos/sin table.
QK_ROPE = [
    ("qkrope_chunk", dict(seed=31, n_q_heads=16, n_kv_heads=8, seq_len=7, start_pos=1000), 4096),
    ("qkrope_decode_32k", dict(seed=32, n_q_heads=32, n_kv_heads=8, seq_len=1, start_pos=32768), 40960),
    ("qkrope_from_zero", dict(seed=33, n_q_heads=4, n_kv_heads=2, seq_len=20, start_pos=0), 64),
]

# Non-paged attention (FlashAttentionImpl<CPU>): (name, seed, B, Hq, Hkv, S,
# causal). Fixtures hold the reference's bf16 output and the inputs' checksums.
FLASH = [
    ("flash_b2_causal", 41, 2, 8, 2, 37, True),
    ("flash_b1_noncausal", 42, 1, 4, 4, 20, False),
]


# KV format export / import: (name, seed, Hkv, [token counts of the
# reference's successive append calls], pool pages). The fixtures hold the
# pages and block table the reference's own append_kv_from_tensor produced,
# checksums of the appended K/V (= the expected bf16 export, regenerated from
# the seed by genllm_b200.synth.kv_format_values), and the expected fp8 export
# (bytes and block scales) computed with numpy fp32 arithmetic and torch's
# float8_e4m3fn conversion.
KV_FORMAT = [
    ("kvfmt_ragged", 51, 2, [21, 16], 8),
    ("kvfmt_heads8", 52, 8, [100, 1, 1, 50], 10),
]
