"""The host tokenizer (b2_tokenizer_*, csrc/tokenizer.cpp) without a GPU.

Parity is checked three ways:
  * golden vectors: tests/golden/tokenizer_{qwen2,llama3,gpt2}.json and the
    ids / decoded text the HF `tokenizers` library gives for 326 strings
    (tests/golden/make_tokenizer_golden.py made them); bit-exact;
  * the live library, where it is importable: seeded adversarial strings
    (combining marks, Hangul jamo, every whitespace kind, contractions in
    every case, special-token fragments, random code points) and NFC over
    every code point; and the character tables regenerated from it;
  * the reference's own tokenizer (src/tokenizer/bpe.cpp, compiled unmodified
    into oracle/_ref/tokenize_ref by oracle/Makefile), which skips the
    vocabulary's NFC normaliser: equal ids wherever the text is already NFC,
    as the reference's own corpus test expects (tests/test_tokenizer.cpp:9-58);
    and the reference's tokenize_stdin app built on this library
    (oracle/_ref/tokenize_b2), equal to the golden ids everywhere.
"""
import ctypes as C
import json
import os
import random
import subprocess
import threading
import unicodedata

import pytest

import b2engine as b2

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
GOLDEN = os.path.join(ROOT, "tests", "golden")
KINDS = ("qwen2", "llama3", "gpt2")


def _path(kind):
    return os.path.join(GOLDEN, f"tokenizer_{kind}.json")


@pytest.fixture(scope="module")
def golden():
    with open(os.path.join(GOLDEN, "tokenizer_cases.json"), encoding="utf-8") as f:
        return json.load(f)


@pytest.fixture(scope="module")
def toks():
    return {k: b2.Tokenizer(_path(k)) for k in KINDS}


@pytest.mark.parametrize("kind", KINDS)
def test_golden_encode(kind, golden, toks):
    t, e = toks[kind], golden["expect"][kind]
    for i, text in enumerate(golden["cases"]):
        assert t.encode(text) == e["ids"][i], (i, text)
        assert t.encode(text, add_special=True) == e["add_special_prefix"] + e["ids"][i], (i, text)
        assert t.encode(text, split_special=False) == e["ids_special_as_text"].get(str(i), e["ids"][i]), (i, text)


@pytest.mark.parametrize("kind", KINDS)
def test_golden_decode(kind, golden, toks):
    t, e = toks[kind], golden["expect"][kind]
    for i, text in enumerate(golden["cases"]):
        want = e["decoded"].get(str(i), text)
        assert t.decode(e["ids"][i]) == want, (i, text)
        assert t.decode(e["ids"][i], skip_special=True) == e["decoded_skip_special"].get(str(i), want), (i, text)


def test_info_and_control_tokens(toks):
    q, l, g = toks["qwen2"], toks["llama3"], toks["gpt2"]
    assert (q.info.pre_tokenizer, q.info.nfc, q.info.ignore_merges, q.info.chat_format) == (1, 1, 0, 1)
    assert (l.info.pre_tokenizer, l.info.nfc, l.info.ignore_merges, l.info.chat_format) == (2, 0, 1, 2)
    assert (g.info.pre_tokenizer, g.info.chat_format) == (3, 0)
    assert q.stop_ids == [q.token_to_id("<|im_end|>"), q.token_to_id("<|endoftext|>")]
    assert l.stop_ids == [l.token_to_id("<|eot_id|>"), l.token_to_id("<|end_of_text|>")]
    assert l.info.bos_id == l.token_to_id("<|begin_of_text|>") and q.info.bos_id == -1
    assert q.info.vocab_size == q.info.n_ids == 2601
    # vocab entries are named as written in tokenizer.json (byte-level symbols)
    assert q.token_to_id("Ġ") == q.encode(" ")[0]
    assert q.token_to_id("no such token") is None


def test_chat_templates(toks):
    msgs = [("system", "You are a helpful assistant."), ("user", "Hello!")]
    # the reference's own expectation (tests/test_tokenizer.cpp:62-66)
    assert toks["qwen2"].apply_chat_template(msgs) == (
        "<|im_start|>system\nYou are a helpful assistant.<|im_end|>\n<|im_start|>user\nHello!<|im_end|>\n"
        "<|im_start|>assistant\n")
    # no system message: the reference's default one (src/tokenizer/bpe.cpp:492-494)
    got = toks["qwen2"].apply_chat_template([{"role": "user", "content": "hi"}], add_generation_prompt=False)
    assert got.startswith("<|im_start|>system\nYou are Qwen,") and got.endswith("<|im_start|>user\nhi<|im_end|>\n")
    # Llama-3: BOS, header / eot per message, contents stripped of surrounding whitespace
    got = toks["llama3"].apply_chat_template([("system", "  Be brief.\n"), ("user", "　Hi there \x1c")])
    assert got == ("<|begin_of_text|><|start_header_id|>system<|end_header_id|>\n\nBe brief.<|eot_id|>"
                   "<|start_header_id|>user<|end_header_id|>\n\nHi there<|eot_id|>"
                   "<|start_header_id|>assistant<|end_header_id|>\n\n")
    ids = toks["llama3"].encode(got)
    assert ids[0] == toks["llama3"].info.bos_id and ids.count(toks["llama3"].token_to_id("<|eot_id|>")) == 2
    with pytest.raises(b2.B2Error):
        toks["gpt2"].apply_chat_template(msgs)


@pytest.mark.parametrize("kind", ("llama3", "gpt2"))
def test_any_bytes_round_trip(kind, toks):
    """Bytes that are not UTF-8 become byte tokens, so decode(encode(x)) == x
    for any byte string (vocabularies without a normaliser)."""
    rng = random.Random(11)
    t = toks[kind]
    for _ in range(400):
        b = bytes(rng.randrange(256) for _ in range(rng.randint(0, 40)))
        assert t.decode_bytes(t.encode(b, split_special=False)) == b


def test_invalid_utf8_kept_under_nfc(toks):
    t = toks["qwen2"]
    b = b"caf\xc3\xa9 \xff\xfe e\xcc\x81 \xe2\x82"
    assert t.decode_bytes(t.encode(b)) == b"caf\xc3\xa9 \xff\xfe \xc3\xa9 \xe2\x82"


def test_errors_and_buffers(toks):
    L = b2.lib()
    # an unknown split pattern, a non-BPE model, malformed JSON, a missing file
    with open(_path("qwen2"), encoding="utf-8") as f:
        d = json.load(f)
    d2 = json.loads(json.dumps(d))
    d2["pre_tokenizer"]["pretokenizers"][0]["pattern"]["Regex"] = r"\w+"
    with pytest.raises(b2.B2Error) as e:
        b2.Tokenizer(json_text=json.dumps(d2))
    assert e.value.status == -2 and "unknown split pattern" in str(e.value)
    d3 = json.loads(json.dumps(d))
    d3["model"]["type"] = "WordPiece"
    with pytest.raises(b2.B2Error) as e:
        b2.Tokenizer(json_text=json.dumps(d3))
    assert e.value.status == -2
    with pytest.raises(b2.B2Error) as e:
        b2.Tokenizer(json_text='{"model": {"vocab": {"a": 0}')
    assert e.value.status == -1
    with pytest.raises(b2.B2Error):
        b2.Tokenizer(os.path.join(GOLDEN, "no_such_tokenizer.json"))
    # an id buffer too small: nothing written, the needed count returned
    t = toks["qwen2"]
    text = b"hello world, hello world"
    n = C.c_size_t(0)
    buf = (C.c_int32 * 2)(-7, -7)
    assert L.b2_tokenizer_encode(t.h, text, len(text), 1, C.cast(buf, C.c_void_p), 2, C.byref(n)) == -3
    assert n.value == len(t.encode(text)) and list(buf) == [-7, -7]
    assert L.b2_tokenizer_encode(None, text, len(text), 1, None, 0, C.byref(n)) == -1
    # empty text, ids outside the vocabulary skipped on decode
    assert t.encode("") == [] and t.decode([-1, 10 ** 6]) == ""


def test_concurrent_encode(toks):
    """A loaded tokenizer is immutable: concurrent encodes agree."""
    rng = random.Random(5)
    texts = ["".join(rng.choice("ab cdéé'S12\n") for _ in range(200)) for _ in range(64)]
    t = toks["qwen2"]
    want = [t.encode(x) for x in texts]
    errs = []

    def work(k):
        for i in range(k, len(texts), 8):
            if t.encode(texts[i]) != want[i]:
                errs.append(i)

    th = [threading.Thread(target=work, args=(k,)) for k in range(8)]
    for x in th:
        x.start()
    for x in th:
        x.join()
    assert not errs


# --- the live HF library -----------------------------------------------------

def _adversarial(rng, n):
    marks = [c for c in range(0x300, 0x20000) if unicodedata.combining(chr(c))]
    alpha = (list(" \t\n\r\x0b\x0c\x85\xa0 　 ") + list("'sStTrReEvVmMlLdDſ")
             + list("0123456789٣४²½") + list(".,!?-_()[]<>|\"#@")
             + [chr(c) for c in marks[:300]] + [chr(c) for c in range(0x1100, 0x1113)]
             + [chr(c) for c in range(0x1161, 0x1176)] + [chr(c) for c in range(0x11A8, 0x11C3)]
             + list("각가한é") + list("aeiouxyzABCXYZαβд中文")
             + ["\U0001f600", "\U0001f44d\U0001f3fd", "‍", "️"]
             + ["<|im_start|>", "<|im_end|>", "<|endoftext|>", "<|eot_id|>", "<|begin_of_text|>", "<mask>",
                "[SEP]", "<tool_call>", "<|im_"])
    out = []
    for _ in range(n):
        s = []
        for _ in range(rng.randint(0, 24)):
            if rng.random() < 0.1:
                c = rng.randrange(1, 0x110000)
                s.append(chr(c if not 0xD800 <= c <= 0xDFFF else 0x41))
            else:
                s.append(rng.choice(alpha))
        out.append("".join(s))
    return out


@pytest.mark.parametrize("kind", KINDS)
def test_live_library_fuzz(kind, toks):
    tk = pytest.importorskip("tokenizers")
    hf = tk.Tokenizer.from_file(_path(kind))
    t = toks[kind]
    strs = _adversarial(random.Random(2026), 6000)
    want = [e.ids for e in hf.encode_batch(strs, add_special_tokens=False)]
    for s, w in zip(strs, want):
        assert t.encode(s) == w, s
    for w in want[:2000]:
        assert t.decode(w) == hf.decode(w, skip_special_tokens=False)
        assert t.decode(w, skip_special=True) == hf.decode(w, skip_special_tokens=True)
    hf.encode_special_tokens = True
    for s, e in zip(strs[:2000], hf.encode_batch(strs[:2000], add_special_tokens=False)):
        assert t.encode(s, split_special=False) == e.ids, s


def test_nfc_every_code_point(toks):
    """decode(encode(x)) of the NFC vocabulary is NFC(x): checked against the
    library's normaliser over every code point, in blocks (so marks meet the
    characters around them)."""
    tk = pytest.importorskip("tokenizers")
    nfc = tk.normalizers.NFC()
    t = toks["qwen2"]
    cps = [c for c in range(1, 0x110000) if not 0xD800 <= c <= 0xDFFF]
    for i in range(0, len(cps), 4096):
        s = "".join(chr(c) for c in cps[i:i + 4096])
        assert t.decode(t.encode(s, split_special=False)) == nfc.normalize_str(s), hex(cps[i])
    rng = random.Random(3)
    marks = [chr(c) for c in range(0x300, 0x370)] + ["ͅ", "ְ", "ཱ", "᷀", "⃐"]
    base = ["a", "e", "o", "ᄀ", "ᅡ", "ᆨ", "가", "Α", "क", "é"]
    for _ in range(3000):
        s = "".join(rng.choice(base if rng.random() < 0.4 else marks) for _ in range(rng.randint(1, 8)))
        assert t.decode(t.encode(s)) == nfc.normalize_str(s), [hex(ord(c)) for c in s]


def test_unicode_tables_regenerate():
    """csrc/unicode_tables.inc is what gen_unicode_tables.py reads off the
    library today."""
    pytest.importorskip("tokenizers")
    import importlib.util
    spec = importlib.util.spec_from_file_location(
        "gen_unicode_tables", os.path.join(ROOT, "serving-engine_b200", "csrc", "gen_unicode_tables.py"))
    gen = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(gen)
    text, _ = gen.build_tables()
    with open(os.path.join(ROOT, "serving-engine_b200", "csrc", "unicode_tables.inc")) as f:
        assert f.read() == text


# --- the reference's tokenizer and its app on this library -------------------

def _stdin_tokenize(exe, tokenizer_json, texts):
    inp = "".join(json.dumps(x) + "\n" for x in texts) + "\n"
    r = subprocess.run([exe, tokenizer_json], input=inp.encode(), capture_output=True, timeout=300)
    assert r.returncode == 0, r.stderr.decode()[-2000:]
    return [json.loads(line) for line in r.stdout.decode().splitlines()]


def _exe(name):
    p = os.path.join(ROOT, "oracle", "_ref", name)
    if not os.path.exists(p):
        pytest.skip(f"oracle/_ref/{name} not built (make -C oracle where the reference sources exist)")
    return p


def test_reference_tokenizer_agrees_on_nfc_text(golden):
    cases = [(i, c) for i, c in enumerate(golden["cases"]) if c]
    got = _stdin_tokenize(_exe("tokenize_ref"), _path("qwen2"), [c for _, c in cases])
    want = golden["expect"]["qwen2"]["ids"]
    stable = 0
    for (i, c), g in zip(cases, got):
        if unicodedata.normalize("NFC", c) == c:
            stable += 1
            assert g == want[i], (i, c)
        else:
            # the reference splits the text as written, without NFC; the
            # golden ids decode to the NFC bytes, so they must differ
            assert g != want[i], (i, c)
    assert stable > 150


def test_reference_app_on_this_library(golden):
    """apps/tokenize_stdin.cpp built against compat/src/tokenizer/bpe.h."""
    cases = [(i, c) for i, c in enumerate(golden["cases"]) if c]
    for kind in KINDS:
        got = _stdin_tokenize(_exe("tokenize_b2"), _path(kind), [c for _, c in cases])
        want = golden["expect"][kind]["ids"]
        assert got == [want[i] for i, _ in cases], kind


def test_reference_tokenizer_is_qwen2_only(golden, tmp_path):
    """What the library adds over the reference's tokenizer: it reads the
    Qwen2 split only (src/tokenizer/bpe.cpp:170-270, one digit per piece, no
    ignore_merges) and merges written as "a b" strings only.  On the Llama-3
    and GPT-2 vocabularies (merges rewritten as strings so that it loads) it
    departs from the HF library on most strings -- digit runs first of all --
    where this library matches every one (test_golden_encode)."""
    exe = _exe("tokenize_ref")
    cases = [(i, c) for i, c in enumerate(golden["cases"]) if c]
    for kind in ("llama3", "gpt2"):
        with open(_path(kind), encoding="utf-8") as f:
            d = json.load(f)
        d["model"]["merges"] = [" ".join(m) if isinstance(m, list) else m for m in d["model"]["merges"]]
        p = tmp_path / f"{kind}_string_merges.json"
        p.write_text(json.dumps(d, ensure_ascii=False), encoding="utf-8")
        got = _stdin_tokenize(exe, str(p), [c for _, c in cases])
        want = golden["expect"][kind]["ids"]
        wrong = [c for (i, c), g in zip(cases, got) if g != want[i]]
        assert len(wrong) > len(cases) // 3, (kind, len(wrong))
        assert "1234" in wrong


def test_single_word_added_tokens_live():
    """single_word added tokens (a match is text when a word character --
    the library's own set, csrc/unicode_tables.inc kWordRanges -- touches
    it), special or not, with rstrip, against the library on seeded strings."""
    tk = pytest.importorskip("tokenizers")
    with open(_path("llama3"), encoding="utf-8") as f:
        d = json.load(f)
    nxt = max(max(d["model"]["vocab"].values()), max(t["id"] for t in d["added_tokens"])) + 1
    for k, (content, special, rstrip) in enumerate([("qqzz", False, False), ("<sw>", True, False),
                                                    ("zq|", False, True)]):
        d["added_tokens"].append({"id": nxt + k, "content": content, "single_word": True, "lstrip": False,
                                  "rstrip": rstrip, "normalized": False, "special": special})
    text = json.dumps(d, ensure_ascii=False)
    t = b2.Tokenizer(json_text=text)
    hf = tk.Tokenizer.from_str(text)
    rng = random.Random(17)
    alpha = (["qqzz", "<sw>", "zq|", "q", "z", "<", ">", "|"] + list("ab_1 \t\n-.é中²ⅷ٣") + ["́", "ǅ", " "])
    strs = ["".join(rng.choice(alpha) for _ in range(rng.randint(1, 10))) for _ in range(4000)]
    strs += ["qqzz", "xqqzz", "qqzzx", "_qqzz", "qqzz_", "²qqzz", "éqqzz", "́qqzz", "a<sw>", " <sw> ",
             "<sw><sw>", "zq|  x", "azq| x", "qqzzqqzz"]
    want = [e.ids for e in hf.encode_batch(strs, add_special_tokens=False)]
    for s, w in zip(strs, want):
        assert t.encode(s) == w, s
    hf.encode_special_tokens = True
    for s, e in zip(strs, hf.encode_batch(strs, add_special_tokens=False)):
        assert t.encode(s, split_special=False) == e.ids, s
