"""HuggingFace checkpoints (safetensors + config.json, optionally tokenizer.json) on CPU: the source
presents them under GGUF names with the same bytes, and the fp32 oracle gives the same logits as on
the GGUF they were converted from (Q/K in rotate-half order with half-rotation RoPE)."""
import json

import numpy as np
import pytest
import torch

from vm_c_b200.gguf.constants import GType
from vm_c_b200.gguf.random_init import preset, write_random_gguf
from vm_c_b200.gguf.reader import GgufSource
from vm_c_b200.hf import HfSource, SafetensorsFile, save_file
from vm_c_b200.hf.source import gguf_name

from hf_convert import gguf_to_hf
from ref_llama import forward_logits, load_dense


def test_safetensors_roundtrip(tmp_path):
    p = str(tmp_path / "a.safetensors")
    t = {"x": torch.randn(3, 5), "y": torch.randn(4, 8).to(torch.bfloat16), "z": torch.arange(7, dtype=torch.int32),
         "h": torch.randn(2, 2).half()}
    save_file(t, p, metadata={"k": "v"})
    f = SafetensorsFile(p)
    assert f.metadata == {"k": "v"}
    assert set(f.entries) == set(t)
    for n, v in t.items():
        raw = np.array(f.raw(n))
        assert raw.tobytes() == v.contiguous().view(torch.uint8).numpy().tobytes(), n
        assert f.entries[n].shape == list(v.shape)
    assert np.array(f.rows_bytes("y", 1, 3)).tobytes() == t["y"][1:3].contiguous().view(torch.uint8).numpy().tobytes()


def test_truncated_file_is_rejected(tmp_path):
    p = tmp_path / "bad.safetensors"
    save_file({"x": torch.randn(16, 16)}, str(p))
    p.write_bytes(p.read_bytes()[:-4])
    with pytest.raises(ValueError):
        SafetensorsFile(str(p))


def test_native_header_parser_edge_cases(tmp_path):
    # Escaped names (\u escapes incl. a surrogate pair, quotes, backslashes), keys the parser must
    # skip (floats, booleans, null, nested values), metadata with escapes, and space padding.
    import struct
    names = ["w\u00e9ight", "emoji_\U0001F600", 'q"uote\\slash']
    data = [np.arange(6, dtype=np.float32).reshape(2, 3), np.arange(4, dtype=np.int32), np.ones(2, np.float16)]
    header, blobs, off = {}, [], 0
    for n, a in zip(names, data):
        b = a.tobytes()
        header[n] = {"dtype": {"float32": "F32", "int32": "I32", "float16": "F16"}[str(a.dtype)], "shape": list(a.shape),
                     "data_offsets": [off, off + len(b)], "extra": {"x": [1.5, True, None, {"y": -2e-3}]}}
        blobs.append(b)
        off += len(b)
    header["__metadata__"] = {"format": "pt", "note": "tab\there \u2603"}
    h = json.dumps(header, ensure_ascii=True).encode() + b"   "
    p = tmp_path / "edge.safetensors"
    p.write_bytes(struct.pack("<Q", len(h)) + h + b"".join(blobs))
    f = SafetensorsFile(str(p))
    assert set(f.entries) == set(names)
    assert f.metadata == {"format": "pt", "note": "tab\there \u2603"}
    for n, a in zip(names, data):
        assert np.array(f.raw(n)).tobytes() == a.tobytes()
    bad = json.dumps({"x": {"dtype": "F32", "shape": [2], "data_offsets": [0, 4]}}).encode()
    p.write_bytes(struct.pack("<Q", len(bad)) + bad + b"\0" * 8)
    with pytest.raises(ValueError):  # byte range does not match the shape
        SafetensorsFile(str(p))
    p.write_bytes(struct.pack("<Q", 5) + b'{"x":')
    with pytest.raises(ValueError):  # truncated JSON
        SafetensorsFile(str(p))



@pytest.mark.parametrize("entry", [
    {"dtype": "F32", "shape": [2 ** 62, 8], "data_offsets": [0, 0]},            # element count overflows
    {"dtype": "F64", "shape": [2 ** 61], "data_offsets": [0, 0]},               # byte size overflows
    {"dtype": "U8", "shape": [8], "data_offsets": [2 ** 63 - 9, 2 ** 63 - 1]},  # range far past the end
    {"dtype": "U8", "shape": [8], "data_offsets": [8, 16]},                     # range just past the end
    {"dtype": "U8", "shape": [-8], "data_offsets": [0, 8]},                     # negative dimension
    {"dtype": "U8", "shape": [8], "data_offsets": [8, 0]},                      # reversed range
])
def test_crafted_header_is_rejected(tmp_path, entry):
    """Sizes and offsets that would wrap 64-bit arithmetic, or reach past the file, are refused while
    the header is read, so no tensor view can point outside the mapped file."""
    import struct
    h = json.dumps({"x": entry}).encode()
    p = tmp_path / "crafted.safetensors"
    p.write_bytes(struct.pack("<Q", len(h)) + h + b"\0" * 8)
    with pytest.raises(ValueError):
        SafetensorsFile(str(p))

def test_name_map():
    assert gguf_name("model.layers.3.self_attn.o_proj.weight") == ("blk.3.attn_output.weight", None)
    assert gguf_name("model.layers.0.block_sparse_moe.experts.5.w2.weight") == ("blk.0.ffn_down_exps.weight", 5)
    assert gguf_name("model.layers.0.self_attn.rotary_emb.inv_freq") is None
    with pytest.raises(ValueError):
        gguf_name("model.layers.0.self_attn.q_proj.bias")


@pytest.mark.parametrize("name", ["tiny-llama", "tiny-mixtral"])
def test_hf_source_matches_gguf(tmp_path, name):
    cfg0 = preset(name)
    gp = str(tmp_path / "m.gguf")
    write_random_gguf(gp, cfg0, "BF16", seed=1)
    g = GgufSource(gp)
    cfg_g = g.model_config()
    hd = tmp_path / "hf"
    gguf_to_hf(g, cfg_g, str(hd))
    h = HfSource(str(hd))
    cfg_h = h.model_config()
    assert cfg_h.rope_neox and not cfg_g.rope_neox
    for f in ("n_layers", "hidden", "n_heads", "n_kv_heads", "head_dim", "ffn", "vocab", "n_experts",
              "n_experts_used", "tie_embeddings"):
        assert getattr(cfg_h, f) == getattr(cfg_g, f), f
    # Same GGUF names and shapes; bytes identical where no permutation applies.
    assert set(h.tensors) == set(g.tensors)
    for n in g.tensors:
        gi, hi = g.info(n), h.info(n)
        assert gi.ne == hi.ne, n
        if gi.gtype == GType.BF16 and "attn_q" not in n and "attn_k" not in n:
            assert hi.gtype == GType.BF16
            assert torch.equal(h.rows(n), g.rows(n)), n
    # Row slices that straddle two experts.
    if cfg_g.is_moe:
        n, F = "blk.1.ffn_up_exps.weight", cfg_g.ffn
        assert torch.equal(h.rows(n, F - 3, F + 5), g.rows(n, F - 3, F + 5))
    rng = np.random.default_rng(0)
    toks = rng.integers(0, cfg_g.vocab, 19).tolist()
    lg = forward_logits(load_dense(g, cfg_g), cfg_g, toks)
    lh = forward_logits(load_dense(h, cfg_h), cfg_h, toks)
    assert torch.allclose(lg, lh, atol=1e-3 * float(lg.abs().max()), rtol=0), float((lg - lh).abs().max())


def test_single_file_and_tied_embeddings(tmp_path):
    cfg = preset("tiny-llama")
    H, V = cfg.hidden, cfg.vocab
    t = {"model.embed_tokens.weight": torch.randn(V, H).bfloat16(), "model.norm.weight": torch.ones(H).bfloat16()}
    d = tmp_path / "m"
    d.mkdir()
    save_file(t, str(d / "model.safetensors"))
    json.dump({"model_type": "llama", "num_hidden_layers": 0, "hidden_size": H, "num_attention_heads": cfg.n_heads,
               "intermediate_size": cfg.ffn, "vocab_size": V}, open(d / "config.json", "w"))
    h = HfSource(str(d / "model.safetensors"))
    assert h.model_config().tie_embeddings
    norm = h.rows("output_norm.weight")
    assert h.info("output_norm.weight").gtype == GType.F32 and norm.dtype == torch.float32
    assert torch.equal(norm.view(-1), torch.ones(H))
    json.dump({"model_type": "qwen2", "num_hidden_layers": 0, "hidden_size": H, "num_attention_heads": 8,
               "intermediate_size": 8, "vocab_size": V}, open(d / "config.json", "w"))
    with pytest.raises(ValueError):
        HfSource(str(d))


def test_tokenizer_json_maps_to_gguf_keys(tmp_path):
    from vm_c_b200.server.tokenizer import Tokenizer, _byte_unicode
    b2u, _ = _byte_unicode()
    alphabet = [b2u[b] for b in range(256)]
    merges = ["h e", "l l", "he ll", "hell o", "Ġ w", "o r", "Ġw or", "Ġwor l", "Ġworl d"]
    tokens = alphabet + [m.replace(" ", "") for m in merges]
    vocab = {t: i for i, t in enumerate(tokens)}
    specials = ["<|begin_of_text|>", "<|end_of_text|>"]
    added = [{"id": len(tokens) + i, "content": s, "special": True} for i, s in enumerate(specials)]
    llama3_split = ("(?i:'s|'t|'re|'ve|'m|'ll|'d)|[^\\r\\n\\p{L}\\p{N}]?\\p{L}+|\\p{N}{1,3}| ?[^\\s\\p{L}\\p{N}]+"
                    "[\\r\\n]*|\\s*[\\r\\n]+|\\s+(?!\\S)|\\s+")
    tj = {"model": {"type": "BPE", "vocab": vocab, "merges": [m.split(" ") for m in merges], "byte_fallback": False},
          "added_tokens": added,
          "pre_tokenizer": {"type": "Sequence", "pretokenizers": [{"type": "Split", "pattern": {"Regex": llama3_split}},
                                                                  {"type": "ByteLevel"}]},
          "post_processor": {"type": "TemplateProcessing", "single": [{"SpecialToken": {"id": "<|begin_of_text|>"}},
                                                                      {"Sequence": {"id": "A"}}]}}
    d = tmp_path / "tok"
    d.mkdir()
    json.dump(tj, open(d / "tokenizer.json", "w"))
    json.dump({"bos_token": "<|begin_of_text|>", "eos_token": {"content": "<|end_of_text|>"},
               "chat_template": "{{ messages[0]['content'] }}"}, open(d / "tokenizer_config.json", "w"))
    V = len(tokens) + 2
    save_file({"model.embed_tokens.weight": torch.zeros(V, 8).bfloat16()}, str(d / "model.safetensors"))
    json.dump({"model_type": "llama", "num_hidden_layers": 0, "hidden_size": 8, "num_attention_heads": 1,
               "intermediate_size": 8, "vocab_size": V}, open(d / "config.json", "w"))
    src = HfSource(str(d))
    assert src.metadata("tokenizer.ggml.pre") == "llama-bpe"
    tok = Tokenizer.from_gguf(src)
    direct = Tokenizer(tokens + specials, [], [1] * len(tokens) + [3, 3], merges, "gpt2", "llama-bpe",
                       len(tokens), [len(tokens) + 1], True, False)
    for text in ["hello world", "hello<|end_of_text|>", " worldhello  x"]:
        assert tok.encode(text) == direct.encode(text), text
        assert tok.decode(tok.encode(text, add_bos=False), skip_special=False) == text
    tokenizers = pytest.importorskip("tokenizers")
    lib_json = {"version": "1.0", "truncation": None, "padding": None, "normalizer": None, "post_processor": None,
                "decoder": None,
                "added_tokens": [dict(a, single_word=False, lstrip=False, rstrip=False, normalized=False) for a in added],
                "pre_tokenizer": {"type": "Sequence", "pretokenizers": [
                    {"type": "Split", "pattern": {"Regex": llama3_split}, "behavior": "Isolated", "invert": False},
                    {"type": "ByteLevel", "add_prefix_space": False, "trim_offsets": True, "use_regex": False}]},
                "model": dict(tj["model"], dropout=None, unk_token=None, continuing_subword_prefix=None,
                              end_of_word_suffix=None, fuse_unk=False, ignore_merges=False)}
    lib = tokenizers.Tokenizer.from_str(json.dumps(lib_json))
    for text in ["hello world", " worldhello  x", "hello\n\nworld 123 héllo"]:
        assert tok.encode(text, add_bos=False) == lib.encode(text, add_special_tokens=False).ids, text
    ids = tok.encode("hello world")
    assert ids[0] == len(tokens)  # BOS from the post-processor template
    assert ids[1:] == [vocab["hello"], vocab["Ġworld"]]
    assert tok.eos_ids == [len(tokens) + 1]
    assert tok.chat_template == "{{ messages[0]['content'] }}"


def test_spm_tokenizer_json_matches_the_tokenizers_library(tmp_path):
    # SentencePiece-style BPE (Llama 2 / Mistral / Mixtral tokenizer.json: byte fallback, "▁" for
    # spaces, a prepended "▁"): our tokenizer built from the mapped keys encodes like the library.
    tokenizers = pytest.importorskip("tokenizers")
    from vm_c_b200.server.tokenizer import Tokenizer
    base = ["<unk>", "<s>", "</s>"] + [f"<0x{b:02X}>" for b in range(256)]
    chars = ["▁"] + list("abcdefghijklmnopqrstuvwxyz") + list(",.!?")
    merges = ["▁ t", "h e", "▁t he", "l l", "he ll", "hell o", "▁ hello", "o r", "▁ w", "▁w or", "l d",
              "▁wor ld", "i n", "▁ in", "▁ a"]
    vocab = {t: i for i, t in enumerate(base + chars)}
    for m in merges:
        a, b = m.split(" ")
        assert a in vocab and b in vocab, m
        vocab.setdefault(a + b, len(vocab))
    tj = {"version": "1.0", "truncation": None, "padding": None,
          "added_tokens": [{"id": i, "content": t, "single_word": False, "lstrip": False, "rstrip": False,
                            "normalized": False, "special": True} for i, t in enumerate(base[:3])],
          "normalizer": {"type": "Sequence", "normalizers": [{"type": "Prepend", "prepend": "▁"},
                                                             {"type": "Replace", "pattern": {"String": " "},
                                                              "content": "▁"}]},
          "pre_tokenizer": None, "post_processor": None, "decoder": None,
          "model": {"type": "BPE", "dropout": None, "unk_token": "<unk>", "continuing_subword_prefix": None,
                    "end_of_word_suffix": None, "fuse_unk": True, "byte_fallback": True, "ignore_merges": False,
                    "vocab": vocab, "merges": [m.split(" ") for m in merges]}}
    d = tmp_path / "spm"
    d.mkdir()
    (d / "tokenizer.json").write_text(json.dumps(tj), encoding="utf-8")
    json.dump({"bos_token": "<s>", "eos_token": "</s>", "add_bos_token": True}, open(d / "tokenizer_config.json", "w"))
    V = len(vocab)
    save_file({"model.embed_tokens.weight": torch.zeros(V, 8).bfloat16()}, str(d / "model.safetensors"))
    json.dump({"model_type": "mistral", "num_hidden_layers": 0, "hidden_size": 8, "num_attention_heads": 1,
               "intermediate_size": 8, "vocab_size": V}, open(d / "config.json", "w"))
    ours = Tokenizer.from_gguf(HfSource(str(d)))
    lib = tokenizers.Tokenizer.from_str(json.dumps(tj))
    for text in ["the world", "hello world in the", "hello, the world!", "a theworld", "héllo wörld", "x  y"]:
        want = lib.encode(text, add_special_tokens=False).ids
        assert ours.encode(text, add_bos=False, parse_special=False) == want, (text, want)
    assert ours.encode("the")[0] == vocab["<s>"]


def test_hf_config_null_fields(tmp_path):
    from vm_c_b200.config import model_config_from_hf
    json.dump({"model_type": "mistral", "num_hidden_layers": 2, "hidden_size": 512, "num_attention_heads": 8,
               "num_key_value_heads": None, "head_dim": None, "intermediate_size": 1024, "vocab_size": 1000,
               "rope_theta": None, "rope_scaling": None, "sliding_window": None}, open(tmp_path / "config.json", "w"))
    m = model_config_from_hf(str(tmp_path))
    assert (m.n_kv_heads, m.head_dim, m.rope_theta, m.rope_scaling) == (8, 64, 10000.0, None) and m.rope_neox
    cfg = json.load(open(tmp_path / "config.json"))
    cfg.update(sliding_window=4096, max_position_embeddings=32768)
    json.dump(cfg, open(tmp_path / "config.json", "w"))
    assert model_config_from_hf(str(tmp_path)).context_length == 4096  # no window mask: capped at the window


def test_hf_config_hybrid_and_nested(tmp_path):
    # Qwen3.5-MoE style: nested text_config, layer_types, linear_* dims, shared expert, partial RoPE.
    from vm_c_b200.config import model_config_from_hf
    tc = {"num_hidden_layers": 8, "hidden_size": 2048, "num_attention_heads": 16, "num_key_value_heads": 2,
          "head_dim": 256, "intermediate_size": 5120, "vocab_size": 151936, "rms_norm_eps": 1e-6,
          "rope_parameters": {"rope_theta": 10000000, "partial_rotary_factor": 0.25}, "num_experts": 256,
          "num_experts_per_tok": 8, "moe_intermediate_size": 512, "shared_expert_intermediate_size": 512,
          "layer_types": (["linear_attention"] * 3 + ["full_attention"]) * 2, "linear_conv_kernel_dim": 4,
          "linear_key_head_dim": 128, "linear_value_head_dim": 128, "linear_num_key_heads": 16,
          "linear_num_value_heads": 32, "max_position_embeddings": 262144}
    json.dump({"model_type": "qwen3_5_moe", "text_config": tc, "eos_token_id": [1, 2]}, open(tmp_path / "config.json", "w"))
    m = model_config_from_hf(str(tmp_path))
    assert m.is_hybrid and m.full_attn_interval == 4
    assert [m.is_recurrent(i) for i in range(8)] == [True, True, True, False] * 2
    assert (m.ssm_conv, m.ssm_state, m.ssm_k_heads, m.ssm_v_heads) == (4, 128, 16, 32)
    assert (m.n_experts, m.n_experts_used, m.ffn, m.ffn_shexp, m.rope_dims) == (256, 8, 512, 512, 64)
    assert m.rope_theta == 10000000 and m.eos_token_ids == [1, 2]
    tc["layer_types"] = ["linear_attention", "full_attention", "linear_attention", "linear_attention"]
    json.dump({"text_config": tc}, open(tmp_path / "config.json", "w"))
    with pytest.raises(ValueError):
        model_config_from_hf(str(tmp_path))


def test_f16_and_f32_weights(tmp_path):
    # F16 matrices are handed over as raw bytes (GGUF F16 rows), F32 matrices as float32 rows.
    H, V = 32, 64
    emb = torch.randn(V, H).half()
    out = torch.randn(V, H)
    save_file({"model.embed_tokens.weight": emb, "lm_head.weight": out, "model.norm.weight": torch.ones(H).half()},
              str(tmp_path / "model.safetensors"))
    json.dump({"model_type": "llama", "num_hidden_layers": 0, "hidden_size": H, "num_attention_heads": 4,
               "intermediate_size": 64, "vocab_size": V}, open(tmp_path / "config.json", "w"))
    h = HfSource(str(tmp_path))
    assert h.info("token_embd.weight").gtype == GType.F16 and h.info("output.weight").gtype == GType.F32
    r = h.rows("token_embd.weight", 3, 7)
    assert r.dtype == torch.uint8 and torch.equal(r.view(torch.float16), emb[3:7])
    assert torch.equal(h.rows("output.weight", 5, 9), out[5:9])
    assert torch.equal(h.rows("output_norm.weight").view(-1), torch.ones(H))


def test_pre_tokenizer_family_from_tokenizer_json():
    """HuggingFace tokenizer.json split expressions map onto the GGUF pre-tokeniser families."""
    from vm_c_b200.hf.source import _pre_family
    from vm_c_b200.server.tokenizer import _PRE
    for fam in ("llama-bpe", "qwen2", "qwen35", "gpt2"):
        pt = {"type": "Sequence", "pretokenizers": [
            {"type": "Split", "pattern": {"Regex": _PRE[fam]}, "behavior": "Isolated", "invert": False},
            {"type": "ByteLevel", "add_prefix_space": False}]}
        assert _pre_family(pt) == fam
    assert _pre_family({"type": "ByteLevel"}) == "gpt2"
