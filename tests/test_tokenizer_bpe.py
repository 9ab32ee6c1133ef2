"""The GGUF byte-level BPE tokenizer (tokenizer.ggml.model = gpt2, the form Llama-3 files
carry: tokens + merges) of csrc/engine/tokenizer.cpp, pinned against the HF tokenizers
library running the same vocabulary with Llama-3's split pattern, byte-level mapping and
ignore_merges.  CPU only."""
import json
import random

import pytest

tk = pytest.importorskip("tokenizers")

LLAMA3_SPLIT = (r"(?i:'s|'t|'re|'ve|'m|'ll|'d)|[^\r\n\p{L}\p{N}]?\p{L}+|\p{N}{1,3}|"
                r" ?[^\s\p{L}\p{N}]+[\r\n]*|\s*[\r\n]+|\s+(?!\S)|\s+")

SPECIALS = ["<|begin_of_text|>", "<|eot_id|>", "<|eot|>", "<|start_header_id|>"]

WORDS = ["hello", "world", "it's", "we'll", "THEY'RE", "naïve", "über", "Straße", "東京", "мир", "123",
         "45678", "3.14", "!!", "...", "x1y2", "café", "don't", "I'M", "e-mail", "(a)", "#tag", "½", "٣٤"]


def _lines(seed, n):
    rng = random.Random(seed)
    seps = [" ", "  ", "\n", " \n", "\t", "\r\n", "   "]
    return ["".join(rng.choice(WORDS) + rng.choice(seps) for _ in range(rng.randint(2, 12))) for _ in range(n)]


@pytest.fixture(scope="module")
def trained(tmp_path_factory):
    from tokenizers import Regex, Tokenizer, decoders, models, pre_tokenizers, trainers
    tok = Tokenizer(models.BPE(ignore_merges=True))
    tok.pre_tokenizer = pre_tokenizers.Sequence([
        pre_tokenizers.Split(Regex(LLAMA3_SPLIT), behavior="isolated", invert=False),
        pre_tokenizers.ByteLevel(add_prefix_space=False, use_regex=False)])
    tok.decoder = decoders.ByteLevel()
    trainer = tk.trainers.BpeTrainer(vocab_size=700, initial_alphabet=pre_tokenizers.ByteLevel.alphabet(),
                                     show_progress=False)
    tok.train_from_iterator(_lines(0, 3000), trainer)
    tok.add_special_tokens(SPECIALS)
    j = json.loads(tok.to_str())
    model = j["model"]
    vocab = dict(model["vocab"])
    for a in j["added_tokens"]:
        vocab[a["content"]] = a["id"]
    pieces = [None] * len(vocab)
    for p, i in vocab.items():
        pieces[i] = p
    types = [3 if p in SPECIALS else 1 for p in pieces]
    merges = [m if isinstance(m, str) else " ".join(m) for m in model["merges"]]
    import vulkangguf as vg
    path = str(tmp_path_factory.mktemp("bpe") / "bpe.gguf")
    vg.write_synthetic_gguf(path, dict(n_layer=1, d_model=256, n_head=4, n_head_kv=4, d_ff=512,
                                       n_vocab=len(pieces), wtype="q4_0", seed=3, vocab=pieces,
                                       scores=[0.0] * len(pieces), token_types=types, merges=merges,
                                       add_bos=False))
    return tok, path


def _texts(seed, n):
    rng = random.Random(seed)
    out = ["", " ", "\n\n", "  x", "a  \n  b", "'s'S'll'LL'd", " 1234567 ", "\t\t!", "end  ", "Ωmega 𝔘nicode 🙂!",
           "tab\tand\r\nCRLF", "x y　z", "ｆｕｌｌ ｗｉｄｔｈ"]
    out += _lines(seed, n)
    for _ in range(n):  # unseen mixtures
        out.append("".join(rng.choice("aZé ñ1٣!?'\n\t.-東😀") for _ in range(rng.randint(1, 30))))
    return out


def test_encode_matches_hf_tokenizers(trained):
    tok, path = trained
    import vulkangguf as vg
    for t in _texts(1, 150):
        want = tok.encode(t).ids
        got = vg.gguf_tokenize(path, t)
        assert got == want, (t, got, want)


def test_special_tokens_in_text_split_out(trained):
    """Control tokens written in the text become their ids (the longest one at each position),
    the text around them is encoded as usual, and decode drops them (as HF's
    skip_special_tokens)."""
    tok, path = trained
    import vulkangguf as vg
    rng = random.Random(4)
    for _ in range(60):
        parts = [rng.choice(WORDS + SPECIALS + [" ", "\n", "<|", "|>", "<|eot"]) for _ in range(rng.randint(1, 10))]
        t = "".join(parts)
        want = tok.encode(t).ids
        ids = vg.gguf_tokenize(path, t)
        assert ids == want, (t, ids, want)
        assert vg.gguf_detokenize(path, ids).decode("utf-8") == tok.decode(ids)


def test_decode_round_trip(trained):
    tok, path = trained
    import vulkangguf as vg
    for t in _texts(2, 80):
        ids = vg.gguf_tokenize(path, t)
        assert vg.gguf_detokenize(path, ids).decode("utf-8") == tok.decode(ids) == t


def test_gpt2_pre_tokenizer_files(tmp_path):
    """tokenizer.ggml.pre = gpt2: GPT-2's own split pattern, merges always applied (no
    ignore_merges), as HF ByteLevel(use_regex=True) with a plain BPE model."""
    from tokenizers import Tokenizer, decoders, models, pre_tokenizers, trainers
    tok = Tokenizer(models.BPE())
    tok.pre_tokenizer = pre_tokenizers.ByteLevel(add_prefix_space=False, use_regex=True)
    tok.decoder = decoders.ByteLevel()
    tok.train_from_iterator(_lines(7, 3000), trainers.BpeTrainer(
        vocab_size=700, initial_alphabet=pre_tokenizers.ByteLevel.alphabet(), show_progress=False))
    model = json.loads(tok.to_str())["model"]
    pieces = [None] * len(model["vocab"])
    for p, i in model["vocab"].items():
        pieces[i] = p
    merges = [m if isinstance(m, str) else " ".join(m) for m in model["merges"]]
    import vulkangguf as vg
    path = str(tmp_path / "gpt2.gguf")
    vg.write_synthetic_gguf(path, dict(n_layer=1, d_model=256, n_head=4, n_head_kv=4, d_ff=512,
                                       n_vocab=len(pieces), wtype="q4_0", seed=3, vocab=pieces,
                                       scores=[0.0] * len(pieces), token_types=[1] * len(pieces), merges=merges,
                                       tokenizer_pre="gpt2", add_bos=False))
    for t in _texts(8, 120):
        want = tok.encode(t).ids
        got = vg.gguf_tokenize(path, t)
        assert got == want, (t, got, want)
        assert vg.gguf_detokenize(path, got).decode("utf-8") == t


def test_unpinned_pre_tokenizer_refused(tmp_path):
    """A byte-level BPE file whose tokenizer.ggml.pre names a split this library does not
    implement (qwen2, deepseek-llm, starcoder, ...) is refused with an error instead of being
    tokenized with the Llama-3 pattern."""
    import vulkangguf as vg
    pieces = [chr(c) for c in range(33, 127)] + ["ab", "abc"]
    path = str(tmp_path / "qwen2-pre.gguf")
    vg.write_synthetic_gguf(path, dict(n_layer=1, d_model=256, n_head=4, n_head_kv=4, d_ff=512,
                                       n_vocab=len(pieces), wtype="q4_0", seed=3, vocab=pieces,
                                       scores=[0.0] * len(pieces), token_types=[1] * len(pieces),
                                       merges=["a b", "ab c"], tokenizer_pre="qwen2", add_bos=False))
    with pytest.raises(Exception) as e:
        vg.gguf_tokenize(path, "abc")
    assert "qwen2" in str(e.value)
