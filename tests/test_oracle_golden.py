"""Pin the CPU oracle to golden vectors produced by the reference's own code."""

import numpy as np
import torch

from oracle import attention, codec, geometry, rope, w8a8
from tests.conftest import bits_to_f32


def test_e4m3_exhaustive_matches_torch():
    b = np.arange(65536, dtype=np.uint32)
    f = codec.bf16_from_bits(b)
    mine = codec.e4m3_encode(f)
    ref = torch.from_numpy(f.copy()).to(torch.bfloat16).to(torch.float8_e4m3fn).view(torch.uint8).numpy()
    nan = np.isnan(f)
    assert np.array_equal(mine[~nan], ref[~nan])
    assert np.array_equal(mine[nan] & 0x7F, ref[nan] & 0x7F)


def test_e4m3_decode_all_codes():
    c = np.arange(256, dtype=np.uint8)
    ref = torch.from_numpy(c.copy()).view(torch.float8_e4m3fn).to(torch.float32).numpy()
    assert np.array_equal(np.nan_to_num(codec.e4m3_decode(c), nan=7e7), np.nan_to_num(ref, nan=7e7))


def test_codec_per_tensor_golden(golden):
    g = golden("codec_per_tensor.npz")
    for i in range(int(g["n"])):
        x = bits_to_f32(g[f"c{i}_x"])
        codes, scale = codec.quant_per_tensor(x)
        assert np.float32(scale) == g[f"c{i}_scale"], i
        assert np.array_equal(codes, g[f"c{i}_codes"]), i
        deq = codec.dequant(codes, scale, per_token=False)
        ref = g[f"c{i}_deq"]
        assert np.array_equal(np.nan_to_num(deq, nan=1e30), np.nan_to_num(ref, nan=1e30)), i


def test_codec_per_token_is_rowwise_per_tensor(golden):
    """Each row of the per-token codec equals the per-tensor codec on that row alone."""
    g = golden("codec_per_tensor.npz")
    for i in range(int(g["n"])):
        x = bits_to_f32(g[f"c{i}_x"])
        x2 = x.reshape(-1, x.shape[-2] * x.shape[-1])
        codes, scales = codec.quant_per_token(x2)
        for r in range(0, x2.shape[0], max(1, x2.shape[0] // 5)):
            c1, s1 = codec.quant_per_tensor(x2[r])
            assert scales[r] == s1 and np.array_equal(codes[r], c1)


def test_w8a8_per_tensor_golden(golden):
    g = golden("w8a8_per_tensor.npz")
    for i in range(int(g["n"])):
        x = bits_to_f32(g[f"c{i}_x"])
        w = bits_to_f32(g[f"c{i}_w"])
        b = bits_to_f32(g[f"c{i}_b"]) if f"c{i}_b" in g else None
        wq, ws = w8a8.quant_weight(w, "e4m3", per_channel=False)
        assert np.float32(ws) == g[f"c{i}_ws"]
        assert np.array_equal(wq, g[f"c{i}_wq"])
        xq, xs = w8a8.quant_act(x, "e4m3", per_token=False)
        y = w8a8.gemm(xq, xs, wq, ws, b, "e4m3")
        ref = bits_to_f32(g[f"c{i}_y"])
        # torch._scaled_mm accumulates in f32; the oracle in f64: same up to one bf16 ulp
        err = np.abs(y - ref).max() / max(np.abs(ref).max(), 1e-6)
        assert err < 1e-2, (i, err)
        assert np.mean(y == ref) > 0.9


def test_rope_golden(golden):
    g = golden("rope.npz")
    for i in range(int(g["n"])):
        f, h, w, sf, n = [int(v) for v in g[f"c{i}_meta"]]
        x = bits_to_f32(g[f"c{i}_x"])
        y = codec.bf16_round(rope.causal_rope_apply(x, f, h, w, sf).astype(np.float32))
        ref = bits_to_f32(g[f"c{i}_y"])
        assert np.array_equal(y, ref), i


def test_geometry_golden(golden):
    recs = golden("geometry.json")
    for r in recs:
        if r["role"] == "denoise":
            gm = geometry.denoise_geometry(r["rank"], r["tick"], r["act_ranks"], r["store_active"],
                                           r["rf_step"], 21, 3, 4680)
            assert gm.naw == r["naw"] and gm.self_off == r["self_off"]
            assert gm.active_len == r["active_len"] and gm.live_off == r["live_off"]
            assert gm.recv_srcs == r["recv_srcs"]
            assert [list(s) for s in gm.send_slots] == r["send_slots"]
            assert gm.active_slots <= r["wmax"]
        elif r["role"] == "store":
            naw, send = geometry.store_geometry(r["tick"], r["act_ranks"], r["rf_step"], 21, 3)
            assert [list(s) for s in send] == r["send_slots"]


def test_tick_roles_cover_schedule(golden):
    recs = golden("geometry.json")
    for r in recs:
        act, csf, qf, st = geometry.tick_roles(r["tick"], r["rf_step"], 12, 3)
        assert act == r["act_ranks"] and csf == r["tick_csf"] and qf == r["tick_qf"]
        assert st == r["store_active"]


def test_sdpa_golden(golden):
    g = golden("sdpa.npz")
    for i in range(int(g["n"])):
        q, k, v = (bits_to_f32(g[f"c{i}_{t}"]) for t in "qkv")
        o = attention.sdpa_numpy(q, k, v)
        ref = g[f"c{i}_o"]
        assert np.abs(o - ref).max() < 1e-5, i


def test_sdpa_numpy_matches_reference_torch_call():
    rng = np.random.default_rng(0)
    q = rng.standard_normal((1, 70, 2, 128)).astype(np.float32)
    k = rng.standard_normal((1, 150, 2, 128)).astype(np.float32)
    v = rng.standard_normal((1, 150, 2, 128)).astype(np.float32)
    ref = attention.sdpa_reference_torch(torch.from_numpy(q), torch.from_numpy(k), torch.from_numpy(v)).numpy()
    o = attention.sdpa_numpy(q[0], k[0], v[0])
    assert np.abs(o - ref[0]).max() < 1e-5


def test_torch_codec_forms_match_the_numpy_restatement(golden):
    """The torch-CPU codec forms (used on config 1's full size) give the numpy
    restatement's codes, scales and dequantised values bit for bit, on the
    golden inputs and on rows with zeros, tiny and large magnitudes."""
    g = golden("codec_per_tensor.npz")
    rng = np.random.default_rng(11)
    mats = []
    for i in range(int(g["n"])):
        x = bits_to_f32(g[f"c{i}_x"])
        mats.append(x.reshape(-1, x.shape[-2] * x.shape[-1]))
    m = codec.bf16_round((rng.standard_normal((64, 256)) * np.exp(rng.uniform(-20, 8, (64, 1)))).astype(np.float32))
    m[3] = 0.0
    m[5, :7] = 1e-30
    mats.append(m)
    for x2 in mats:
        xt = torch.from_numpy(np.ascontiguousarray(x2)).to(torch.bfloat16)
        c_ref, s_ref = codec.quant_per_tensor(x2)
        c, s = codec.quant_per_tensor_torch(xt)
        assert float(s) == float(s_ref) and np.array_equal(c.numpy(), c_ref)
        d = codec.dequant_torch(c, s, per_token=False).numpy()
        assert np.array_equal(np.nan_to_num(d, nan=1e30),
                              np.nan_to_num(codec.dequant(c_ref, s_ref, per_token=False), nan=1e30))
        c_ref, s_ref = codec.quant_per_token(x2)
        c, s = codec.quant_per_token_torch(xt)
        assert np.array_equal(s.numpy(), s_ref) and np.array_equal(c.numpy(), c_ref)
        d = codec.dequant_torch(c, s, per_token=True).numpy()
        assert np.array_equal(np.nan_to_num(d, nan=1e30),
                              np.nan_to_num(codec.dequant(c_ref, s_ref, per_token=True), nan=1e30))
