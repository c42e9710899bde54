"""Writes .qint8 files for the loader tests: the on-disk layout of
write_qint8_v2_file (crates/qwen-asr/src/quantize.rs:481-590) restated --
magic "QINT8\\x02\\0\\0", tensor count, reserved word, then per tensor
(name_len u16, name, dtype u8, n_dims u8, shape u32 x n_dims, data offset
u64, scale offset u64), then the data section: INT8 tensors first (bytes,
zero padding to 4, f32 scales), then F32 tensors (4-aligned), then BF16
(2-aligned); offsets are relative to the start of the data section.  With
version=1 the dtype byte is omitted (V1 infers it from the scale offset).

Tensor names follow qwen-asr-quantize (crates/qwen-asr-quantize/src/main.rs)
and the loaders (decoder.rs:680-748, encoder.rs:466-520).
"""
from __future__ import annotations

import struct

import numpy as np

INT8, F32, BF16 = 0, 1, 2


def write_qint8(path, entries, version=2):
    """entries: list of (name, dtype, array, scales-or-None)."""
    data = bytearray()
    table = []
    order = [e for e in entries if e[1] == INT8] + [e for e in entries if e[1] == F32] + \
        [e for e in entries if e[1] == BF16]
    for name, dt, arr, sc in order:
        arr = np.ascontiguousarray(arr)
        if dt == INT8:
            off = len(data)
            data += arr.astype(np.int8).tobytes()
            while len(data) % 4:
                data.append(0)
            soff = len(data)
            data += np.asarray(sc, np.float32).tobytes()
        elif dt == F32:
            while len(data) % 4:
                data.append(0)
            off, soff = len(data), 0
            data += arr.astype(np.float32).tobytes()
        else:
            while len(data) % 2:
                data.append(0)
            off, soff = len(data), 0
            data += arr.astype(np.uint16).tobytes()
        table.append((name, dt, arr.shape, off, soff))
    with open(path, "wb") as f:
        f.write(b"QINT8" + bytes([version, 0, 0]))
        f.write(struct.pack("<II", len(table), 0))
        for name, dt, shape, off, soff in table:
            nb = name.encode()
            f.write(struct.pack("<H", len(nb)) + nb)
            if version == 2:
                f.write(bytes([dt]))
            f.write(bytes([len(shape)]))
            for d in shape:
                f.write(struct.pack("<I", d))
            f.write(struct.pack("<QQ", off, soff))
        f.write(bytes(data))


def bf16_bits(a):
    """Truncating f32 -> bf16 (the high 16 bits)."""
    return (np.asarray(a, np.float32).view(np.uint32) >> 16).astype(np.uint16)


def model_entries(dec_w, enc_w=None, int8_embed=None, with_lm_head=True):
    """Tensor entries of a V2 file from synthetic weights: dec_w from
    synthetic.decoder_weights_np (gate/up stored interleaved there, split back
    into gate_proj / up_proj here), enc_w in the INT8 form of
    synthetic.quantize_encoder.  int8_embed = (table, scales) for an INT8
    embedding table (V2 files carry one); otherwise the f32 table is written."""
    e = []
    p = "thinker.model."
    for i, L in enumerate(dec_w["layers"]):
        lp = f"{p}layers.{i}."
        for n, k in (("self_attn.q_proj", "wq"), ("self_attn.k_proj", "wk"), ("self_attn.v_proj", "wv"),
                     ("self_attn.o_proj", "wo"), ("mlp.down_proj", "down")):
            e.append((lp + n + ".weight", INT8, L[k], L[k + "_s"]))
        e.append((lp + "mlp.gate_proj.weight", INT8, L["gate_up"][0::2], L["gate_up_s"][0::2]))
        e.append((lp + "mlp.up_proj.weight", INT8, L["gate_up"][1::2], L["gate_up_s"][1::2]))
        for n, k in (("self_attn.q_norm", "q_norm"), ("self_attn.k_norm", "k_norm"),
                     ("input_layernorm", "input_norm"), ("post_attention_layernorm", "post_attn_norm")):
            e.append((lp + n + ".weight", F32, L[k], None))
    e.append((p + "norm.weight", F32, dec_w["norm"], None))
    if int8_embed is not None:
        e.append((p + "embed_tokens.weight", INT8, int8_embed[0], int8_embed[1]))
    else:
        e.append((p + "embed_tokens.weight", F32, dec_w["embed"], None))
    if with_lm_head:
        e.append(("thinker.lm_head.weight", INT8, dec_w["lm_head"], dec_w["lm_head_s"]))
    if enc_w is not None:
        a = "thinker.audio_tower."
        for c in (1, 2, 3):
            e.append((f"{a}conv2d{c}.weight", F32, enc_w[f"conv{c}_w"], None))
            e.append((f"{a}conv2d{c}.bias", F32, enc_w[f"conv{c}_b"], None))
        e.append((a + "conv_out.weight", INT8, enc_w["conv_out"], enc_w["conv_out_s"]))
        for i, L in enumerate(enc_w["layers"]):
            lp = f"{a}layers.{i}."
            for n, k, b in (("self_attn.q_proj", "wq", "bq"), ("self_attn.k_proj", "wk", "bk"),
                            ("self_attn.v_proj", "wv", "bv"), ("self_attn.out_proj", "wo", "bo"),
                            ("fc1", "fc1", "fc1_b"), ("fc2", "fc2", "fc2_b")):
                e.append((lp + n + ".weight", INT8, L[k], L[k + "_s"]))
                e.append((lp + n + ".bias", F32, L[b], None))
            for n, k in (("self_attn_layer_norm.weight", "attn_norm_w"), ("self_attn_layer_norm.bias", "attn_norm_b"),
                         ("final_layer_norm.weight", "ffn_norm_w"), ("final_layer_norm.bias", "ffn_norm_b")):
                e.append((lp + n, F32, L[k], None))
        for n in ("ln_post.weight", "ln_post.bias", "proj1.bias", "proj2.bias"):
            e.append((a + n, F32, enc_w[n.replace(".weight", "_w").replace(".bias", "_b")], None))
        for n in ("proj1", "proj2"):
            e.append((a + n + ".weight", INT8, enc_w[n], enc_w[n + "_s"]))
    return e
