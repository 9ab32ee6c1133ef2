"""The GGUF SentencePiece tokenizer of the text surface (csrc/engine/tokenizer.cpp), pinned
against the sentencepiece library on a BPE model trained here with LLaMA's tokenizer settings
(identity normaliser, dummy-prefix space, byte fallback) and written into a synthetic GGUF as
tokenizer.ggml.{tokens, scores, token_type} -- the form llama.cpp's files carry it in.

CPU only: the tokenizer is host code and no model is loaded."""
import io
import random

import pytest

spm = pytest.importorskip("sentencepiece")

ALPHABET = "abcdefghijklmnopqrstuvwxyz" + "éüß" + "0123456789"


def _corpus(seed=0, n_lines=3000):
    rng = random.Random(seed)
    words = ["".join(rng.choice(ALPHABET) for _ in range(rng.randint(1, 9))) for _ in range(400)]
    return [" ".join(rng.choice(words) for _ in range(rng.randint(3, 14))) for _ in range(n_lines)], words


@pytest.fixture(scope="module")
def trained(tmp_path_factory):
    lines, words = _corpus()
    buf = io.BytesIO()
    spm.SentencePieceTrainer.train(sentence_iterator=iter(lines), model_writer=buf, vocab_size=600,
                                   model_type="bpe", byte_fallback=True, normalization_rule_name="identity",
                                   add_dummy_prefix=True, remove_extra_whitespaces=False, split_digits=True,
                                   minloglevel=2)
    sp = spm.SentencePieceProcessor(model_proto=buf.getvalue())
    n = sp.get_piece_size()
    pieces = [sp.id_to_piece(i) for i in range(n)]
    scores = [sp.get_score(i) for i in range(n)]

    def ttype(i):
        if sp.is_unknown(i):
            return 2
        if sp.is_control(i):
            return 3
        if sp.is_byte(i):
            return 6
        if sp.is_unused(i):
            return 5
        return 1

    types = [ttype(i) for i in range(n)]
    import vulkangguf as vg
    path = str(tmp_path_factory.mktemp("tok") / "vocab.gguf")
    vg.write_synthetic_gguf(path, dict(n_layer=1, d_model=256, n_head=4, n_head_kv=4, d_ff=512, n_vocab=n,
                                       wtype="q4_0", seed=3, vocab=pieces, scores=scores, token_types=types))
    return sp, path, words


def _texts(words, seed=1, n=200):
    rng = random.Random(seed)
    out = ["", " ", "a", "  leading and  double  spaces ", "trailing ", "€ and 中文 are not in the corpus",
           "tab\tand\nnewline", "0123456789 9876"]
    for _ in range(n):
        k = rng.randint(1, 12)
        parts = []
        for _ in range(k):
            r = rng.random()
            if r < 0.7:
                parts.append(rng.choice(words))
            elif r < 0.85:  # unseen spellings of seen characters
                parts.append("".join(rng.choice(ALPHABET) for _ in range(rng.randint(1, 12))))
            else:  # characters outside the vocabulary: byte fallback
                parts.append(rng.choice(["€", "Ω", "ж", "🙂", "~", "ÿ"]) * rng.randint(1, 3))
        out.append((" " * rng.randint(1, 2)).join(parts))
    return out


def test_encode_matches_sentencepiece(trained):
    sp, path, words = trained
    import vulkangguf as vg
    for t in _texts(words):
        want = sp.encode(t) if t else []
        got = vg.gguf_tokenize(path, t, add_bos=False)
        assert got == want, (t, got, want)


def test_bos_and_decode_round_trip(trained):
    sp, path, words = trained
    import vulkangguf as vg
    for t in _texts(words, seed=2, n=100):
        ids = vg.gguf_tokenize(path, t)  # the file has no add_bos_token key: BOS by default
        assert ids[0] == 1  # <s>
        assert vg.gguf_detokenize(path, ids).decode("utf-8") == sp.decode(ids[1:]) == t


def test_decode_of_random_ids_matches_sentencepiece(trained):
    """Any id sequence (byte runs that are not valid UTF-8, control and unknown ids included)
    decodes as sentencepiece decodes it."""
    sp, path, words = trained
    import vulkangguf as vg
    rng = random.Random(3)
    n = sp.get_piece_size()
    for _ in range(300):
        ids = [rng.randrange(n) for _ in range(rng.randint(1, 20))]
        assert vg.gguf_detokenize(path, ids).decode("utf-8") == sp.decode(ids), ids


def test_file_flags_no_space_prefix_and_no_bos(tmp_path):
    """A file with tokenizer.ggml.add_space_prefix = false encodes without the dummy prefix
    (as sentencepiece with add_dummy_prefix=False) and keeps a leading space on decode; with
    add_bos_token = false, add_bos=None prepends no BOS."""
    lines, words = _corpus(seed=5, n_lines=2000)
    buf = io.BytesIO()
    spm.SentencePieceTrainer.train(sentence_iterator=iter(lines), model_writer=buf, vocab_size=500,
                                   model_type="bpe", byte_fallback=True, normalization_rule_name="identity",
                                   add_dummy_prefix=False, remove_extra_whitespaces=False, minloglevel=2)
    sp = spm.SentencePieceProcessor(model_proto=buf.getvalue())
    n = sp.get_piece_size()
    types = [2 if sp.is_unknown(i) else 3 if sp.is_control(i) else 6 if sp.is_byte(i) else 1 for i in range(n)]
    import vulkangguf as vg
    path = str(tmp_path / "noprefix.gguf")
    vg.write_synthetic_gguf(path, dict(n_layer=1, d_model=256, n_head=4, n_head_kv=4, d_ff=512, n_vocab=n,
                                       wtype="q4_0", seed=3, vocab=[sp.id_to_piece(i) for i in range(n)],
                                       scores=[sp.get_score(i) for i in range(n)], token_types=types,
                                       add_bos=False, add_space_prefix=False))
    for t in _texts(words, seed=6, n=100) + [" leading space", "  two"]:
        ids = vg.gguf_tokenize(path, t)
        assert ids == (sp.encode(t) if t else []), t
        assert vg.gguf_detokenize(path, ids).decode("utf-8") == sp.decode(ids) == t


def test_gguf_without_vocabulary_is_rejected(tmp_path):
    import vulkangguf as vg
    p = str(tmp_path / "novocab.gguf")
    vg.write_synthetic_gguf(p, dict(n_layer=1, d_model=256, n_head=4, n_head_kv=4, d_ff=512, n_vocab=512,
                                    wtype="q4_0", seed=3))
    with pytest.raises(RuntimeError, match="vocabulary"):
        vg.gguf_tokenize(p, "abc")


@pytest.mark.gpu
def test_generate_text_uses_the_gguf_vocabulary(trained):
    """InferenceAPI.generate(str) on a model whose GGUF carries the vocabulary: the prompt is
    encoded with it (BOS first) and the continuation decoded with it."""
    sp, path, words = trained
    import vulkangguf as vg
    api = vg.InferenceAPI()
    assert api.load_model(path)
    cfg = vg.GenerationConfig()
    cfg.max_tokens = 12
    cfg.temperature = 0.0
    cfg.do_sample = False
    prompt = " ".join(words[:6])
    ids = vg.gguf_tokenize(path, prompt, True)
    toks = api.generate_tokens(ids, cfg)
    assert api.generate(prompt, cfg) == sp.decode(list(toks))


def test_truncated_vocabulary_arrays_rejected(trained, tmp_path):
    """A GGUF cut inside its tokenizer arrays is rejected with an error, never read past its end."""
    sp, path, words = trained
    import vulkangguf as vg
    data = open(path, "rb").read()
    cut = data.find(b"tokenizer.ggml.scores")
    assert cut > 0
    bad = str(tmp_path / "cut.gguf")
    for n in (cut - 100, cut + 30):
        with open(bad, "wb") as f:
            f.write(data[:n])
        with pytest.raises(RuntimeError):
            vg.gguf_tokenize(bad, "abc")


def test_user_defined_pieces_match_first_and_never_merge(tmp_path):
    """User-defined pieces (the added symbols of fine-tuned vocabularies) are matched first,
    longest at each position, and never merged with their neighbours, as sentencepiece does."""
    rng = random.Random(0)
    alpha = "abcdefghijklmnopqrstuvwxyz"
    words = ["".join(rng.choice(alpha) for _ in range(rng.randint(1, 8))) for _ in range(300)]
    lines = [" ".join(rng.choice(words) for _ in range(10)) for _ in range(2000)]
    user = ["<tool>", "ab", "xyz"]
    buf = io.BytesIO()
    spm.SentencePieceTrainer.train(sentence_iterator=iter(lines), model_writer=buf, vocab_size=500, model_type="bpe",
                                   byte_fallback=True, normalization_rule_name="identity", add_dummy_prefix=True,
                                   remove_extra_whitespaces=False, user_defined_symbols=user, minloglevel=2)
    sp = spm.SentencePieceProcessor(model_proto=buf.getvalue())
    n = sp.get_piece_size()

    def ttype(i):
        if sp.is_unknown(i):
            return 2
        if sp.is_control(i):
            return 3
        if sp.is_byte(i):
            return 6
        return 4 if sp.id_to_piece(i) in user else 1

    import vulkangguf as vg
    path = str(tmp_path / "user.gguf")
    vg.write_synthetic_gguf(path, dict(n_layer=1, d_model=256, n_head=4, n_head_kv=4, d_ff=512, n_vocab=n,
                                       wtype="q4_0", seed=3, vocab=[sp.id_to_piece(i) for i in range(n)],
                                       scores=[sp.get_score(i) for i in range(n)],
                                       token_types=[ttype(i) for i in range(n)]))
    for _ in range(300):
        t = " ".join(rng.choice(words + ["<tool>", "ab", "xyzab", "aab", "<tool>x"]) for _ in range(rng.randint(1, 8)))
        if rng.random() < 0.3:
            t = t.replace(" ", "")
        assert vg.gguf_tokenize(path, t, add_bos=False) == sp.encode(t), t
