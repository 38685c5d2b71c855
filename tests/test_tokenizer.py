"""Tokenizer (GGUF vocab, native BPE core), incremental detokenizer, chat template, reasoning split."""
import pytest

from vm_c_b200.gguf.random_init import preset, synthetic_vocab, write_random_gguf
from vm_c_b200.gguf.reader import GgufSource
from vm_c_b200.server.chat import ChatTemplate, ReasoningStream, chatml, split_reasoning
from vm_c_b200.server.tokenizer import IncrementalDetokenizer, Tokenizer, _byte_unicode


def spm_tok():
    toks, scores, types = synthetic_vocab(2000)
    # give merged pieces higher scores than their parts
    scores = [float(len(t)) if ty == 1 else 0.0 for t, ty in zip(toks, types)]
    return Tokenizer(toks, scores, types, [], "llama", "gpt2", 1, [2], True)


def test_spm_roundtrip_ascii_and_bytes():
    tok = spm_tok()
    for text in ["hello world", "the rain in spain", "naïve café ☃ 漢字", "a\nb\tc"]:
        ids = tok.encode(text)
        assert ids[0] == 1
        assert tok.decode(ids).lstrip() == text
    # merges happen: "▁th" style pieces exist in the synthetic vocab
    assert len(tok.encode("tete", add_bos=False)) < 4


def gpt2_tok():
    b2u, _ = _byte_unicode()
    toks = [b2u[b] for b in range(256)]
    merges = []
    for a, b in [("h", "e"), ("l", "l"), ("he", "ll"), ("Ġ", "w"), ("o", "r"), ("Ġw", "or"), ("l", "d")]:
        merges.append(f"{a} {b}")
        toks.append(a + b)
    toks += ["<|bos|>", "<|eot|>"]
    types = [1] * (len(toks) - 2) + [3, 3]
    return Tokenizer(toks, [], types, merges, "gpt2", "llama-bpe", len(toks) - 2, [len(toks) - 1], True)


def test_gpt2_bpe_merges_and_specials():
    tok = gpt2_tok()
    ids = tok.encode("hello world<|eot|>", add_bos=False)
    pieces = [tok.tokens[i] for i in ids]
    assert pieces == ["hell", "o", "Ġwor", "ld", "<|eot|>"]
    assert tok.decode(ids) == "hello world"
    assert tok.decode(ids, skip_special=False) == "hello world<|eot|>"
    assert tok.decode(tok.encode("ünï", add_bos=False)) == "ünï"


def test_incremental_detokenizer_utf8_and_stop():
    tok = gpt2_tok()
    ids = tok.encode("héllo world", add_bos=False)
    d = IncrementalDetokenizer(tok)
    out = "".join(d.push([i]) for i in ids) + d.push([], final=True)
    assert out == "héllo world"
    d = IncrementalDetokenizer(tok, stop=["wor"])
    out = "".join(d.push([i]) for i in ids)
    assert out == "héllo " and d.stopped


def test_tokenizer_from_random_gguf(tmp_path):
    p = tmp_path / "t.gguf"
    write_random_gguf(str(p), preset("tiny-llama"), "Q8_0", seed=0)
    tok = Tokenizer.from_gguf(GgufSource(str(p)))
    assert tok.vocab_size == 32000 and tok.bos_id == 1 and tok.eos_ids == [2]
    assert tok.decode(tok.encode("some text here")).strip() == "some text here"


def test_chat_template_fallback_and_jinja():
    msgs = [{"role": "system", "content": "S"}, {"role": "user", "content": "U"}]
    p = ChatTemplate(None).render(msgs, True, True)
    assert p == "<|im_start|>system\nS<|im_end|>\n<|im_start|>user\nU<|im_end|>\n<|im_start|>assistant\n<think>\n"
    assert chatml(msgs, True, False).endswith("<think>\n\n</think>\n\n")
    t = ChatTemplate("{% for m in messages %}[{{ m.role }}]{{ m.content }}{% endfor %}"
                     "{% if add_generation_prompt %}[assistant]{% endif %}")
    assert t.render(msgs) == "[system]S[user]U[assistant]"


def test_reasoning_split():
    assert split_reasoning("think hard</think>\n\nanswer", True) == ("think hard", "answer")
    assert split_reasoning("no tags", True) == ("", "no tags")
    rs = ReasoningStream(True)
    got = [rs.feed(x) for x in ["abc</th", "ink>", "\n", "ans", "wer"]]
    reasoning = "".join(r for r, _ in got)
    content = "".join(c for _, c in got)
    assert reasoning == "abc" and content == "answer"
