"""Makes the tokenizer fixtures: three small byte-level BPE tokenizer.json
files trained with the HF `tokenizers` library on seeded synthetic text, and
the ids / decoded text that library gives for a set of test strings.

  tokenizer_qwen2.json   NFC normaliser, the Qwen2 split pattern (one digit per
                         piece), merges written as "a b" strings (the form the
                         reference's loader reads, src/tokenizer/bpe.cpp:128-135),
                         ChatML control tokens, one non-special added token
  tokenizer_llama3.json  no normaliser, the Llama-3 split pattern (up to three
                         digits), ignore_merges, <|begin_of_text|> added by a
                         TemplateProcessing post-processor, merges as [a, b]
  tokenizer_gpt2.json    ByteLevel with its own regex, <|endoftext|>, added
                         tokens with lstrip / rstrip and one matched after
                         normalisation
  tokenizer_cases.json   per tokenizer and test string: ids (plain, with the
                         post-processor, with special tokens read as text) and
                         the decoded text (with and without special tokens)

The training text and the test strings are generated here from fixed seeds
(mixed scripts, combining marks in composed and decomposed form, digits,
contractions, whitespace runs, code, emoji); no external data.

Usage: python tests/golden/make_tokenizer_golden.py
"""
import json
import os
import random

from tokenizers import AddedToken, Regex, Tokenizer, decoders, models, normalizers, pre_tokenizers, processors, trainers

HERE = os.path.dirname(os.path.abspath(__file__))

QWEN2 = r"(?i:'s|'t|'re|'ve|'m|'ll|'d)|[^\r\n\p{L}\p{N}]?\p{L}+|\p{N}| ?[^\s\p{L}\p{N}]+[\r\n]*|\s*[\r\n]+|\s+(?!\S)|\s+"
LLAMA3 = r"(?i:'s|'t|'re|'ve|'m|'ll|'d)|[^\r\n\p{L}\p{N}]?\p{L}+|\p{N}{1,3}| ?[^\s\p{L}\p{N}]+[\r\n]*|\s*[\r\n]+|\s+(?!\S)|\s+"

SYLLABLES = {
    "latin": ["ka", "to", "ri", "men", "sal", "ber", "qu", "th", "ing", "ed", "str", "on", "ar", "el", "is",
              "and", "the", "of", "ex", "pre", "con", "ly", "tion", "X", "Z", "Be", "Ma"],
    "accent": ["é", "è", "ü", "ñ", "ç", "å", "ø", "ß", "é", "ä", "ộ", "ǖ", "Å", "ő"],
    "greek": ["αλ", "φα", "βη", "τα", "ου", "ζω", "ή", "ώ", "ΘΕ"],
    "cyrillic": ["при", "вет", "мир", "ка", "ть", "ЖИ", "щ", "ё"],
    "cjk": ["中", "文", "字", "語", "日本", "人", "大", "学", "東京", "的", "是"],
    "hangul": ["한", "국", "어", "서울", "가", "한"],
    "arabic": ["مر", "حبا", "سلا", "م", "ال"],
    "devanagari": ["नम", "स्ते", "हि", "न्दी", "क्ष"],
}
EMOJI = ["😀", "👍🏽", "👨‍👩‍👧", "🇯🇵", "✨", "❤️"]
PUNCT = [".", ",", "!", "?", ";", ":", "...", "—", "(", ")", "[", "]", "{", "}", "\"", "'", "«", "»", "#", "@",
         "$", "%", "&", "*", "+", "=", "<", ">", "/", "\\", "|", "~", "`", "^", "_", "-", "→", "©", "½", "²"]
SPACES = [" ", " ", " ", " ", "  ", "\t", "\n", "\n\n", "\r\n", " \n", " ", "　", "   ", " ", "\x0b"]
CONTRACTIONS = ["'s", "'t", "'re", "'ve", "'m", "'ll", "'d", "'S", "'T", "'RE", "'Ve", "'LL", "'D", "'ſ", "'x"]


def word(rng):
    script = rng.choice(list(SYLLABLES))
    w = "".join(rng.choice(SYLLABLES[script]) for _ in range(rng.randint(1, 4)))
    r = rng.random()
    if r < 0.08:
        w += rng.choice(CONTRACTIONS)
    elif r < 0.16:
        w = w.capitalize()
    return w


def number(rng):
    return "".join(rng.choice("0123456789٣४") if rng.random() < 0.05 else rng.choice("0123456789")
                   for _ in range(rng.randint(1, 9)))


def code_line(rng):
    ind = " " * rng.choice([0, 2, 4, 8])
    name = "".join(rng.choice("abcdefxyz_") for _ in range(rng.randint(1, 8)))
    forms = [f"{ind}def {name}(x, y={rng.randint(0, 99)}):", f"{ind}return {name}[{rng.randint(0, 9)}] + 1;",
             f"{ind}if ({name} != NULL) {{", f"{ind}}}", f"{ind}// {name} -- note", f"{ind}{name} = \"{word(rng)}\""]
    return rng.choice(forms)


def text(rng, n):
    out = []
    for _ in range(n):
        r = rng.random()
        if r < 0.55:
            out.append(word(rng))
        elif r < 0.65:
            out.append(number(rng))
        elif r < 0.77:
            out.append(rng.choice(PUNCT))
        elif r < 0.80:
            out.append(rng.choice(EMOJI))
        elif r < 0.84:
            out.append("\n" + code_line(rng) + "\n")
        out.append(rng.choice(SPACES) if rng.random() < 0.4 else " ")
    return "".join(out)


def edge_cases():
    cases = ["", " ", "a", "  ", "\n", "\r\n", "\t\t", "   x", "x   ", "x   y", "x \n y", " \n\n ",
             "hello world", "Hello, World!", "don't", "DON'T", "we're", "they'VE", "I'm", "you'll", "he'd",
             "it'ſ", "'s", "''", "'", "'''s", "x's'", "1", "12", "123", "1234", "1234567", "3.14159",
             "version 2.0.1-rc3", "$1,000,000", "٣٤٥", "४२", "²³", "½", "x́", "é", "é", "ẹ́",
             "ẹ́", "각", "각", "Å", "Å", "Å", "ﬁ", "ｆｕｌｌ", "Ωmega",
             "中文字符测试", "日本語のテキスト", "한국어 텍스트", "مرحبا بالعالم", "नमस्ते दुनिया", "Привет, мир!",
             "😀😀😀", "👨‍👩‍👧 family", "🇯🇵🇫🇷", "a b", "a　b", "a b", "tab\there",
             "line1\nline2\r\nline3\rline4", "    indented\n        more", "trailing   ", "\n\n\nx", "x\n\n\n",
             "def f(x):\n    return x + 1\n", "if (a != b) { c = d; }", "<html><body>hi</body></html>",
             "a" * 300, "ab" * 150, " " * 50, "\n" * 20, "!?" * 40, "0" * 40,
             "<|im_start|>user\nhi<|im_end|>", "<|im_start|><|im_end|>", "<|im_sta", "<|endoftext|>x<|endoftext|>",
             "x<|im_end|>y", "<|begin_of_text|>Hello", "<|start_header_id|>system<|end_header_id|>\n\nhi<|eot_id|>",
             "<|eot_id|><|eot_id|>", "text <tool_call> more", "<tool_call>", "  <mask>  x", "a<mask>b",
             "[SEP] next", "x [SEP]y", "😀<|endoftext|>😀", "́start", "endś", "̀ͅ",
             "ſ", "K", "İstanbul", "ß", "ǅ", "x​x", "﻿bom", "\x00nul\x01", "\x7f\x80\x9f"]
    return cases


def train(kind, corpus):
    specials = {
        "qwen2": ["<|endoftext|>", "<|im_start|>", "<|im_end|>"],
        "llama3": ["<|begin_of_text|>", "<|end_of_text|>", "<|start_header_id|>", "<|end_header_id|>",
                   "<|eot_id|>", "<|reserved_special_token_0|>", "<|reserved_special_token_1|>"],
        "gpt2": ["<|endoftext|>"],
    }[kind]
    tok = Tokenizer(models.BPE(ignore_merges=(kind == "llama3")))
    if kind == "qwen2":
        tok.normalizer = normalizers.NFC()
    if kind == "gpt2":
        tok.pre_tokenizer = pre_tokenizers.ByteLevel(add_prefix_space=False, use_regex=True)
    else:
        tok.pre_tokenizer = pre_tokenizers.Sequence([
            pre_tokenizers.Split(Regex(QWEN2 if kind == "qwen2" else LLAMA3), behavior="isolated"),
            pre_tokenizers.ByteLevel(add_prefix_space=False, use_regex=False),
        ])
    tok.decoder = decoders.ByteLevel()
    trainer = trainers.BpeTrainer(vocab_size=2600, min_frequency=2, show_progress=False,
                                  initial_alphabet=pre_tokenizers.ByteLevel.alphabet(),
                                  special_tokens=[AddedToken(s, special=True, normalized=False) for s in specials])
    tok.train_from_iterator(corpus, trainer=trainer)
    if kind == "qwen2":
        tok.add_tokens([AddedToken("<tool_call>", special=False, normalized=False)])
        tok.post_processor = processors.ByteLevel(trim_offsets=False)
    elif kind == "llama3":
        bos = tok.token_to_id("<|begin_of_text|>")
        tok.post_processor = processors.Sequence([
            processors.ByteLevel(trim_offsets=True),
            processors.TemplateProcessing(single="<|begin_of_text|> $A", pair="<|begin_of_text|> $A $B:1",
                                          special_tokens=[("<|begin_of_text|>", bos)]),
        ])
    else:
        tok.add_tokens([AddedToken("<mask>", special=True, lstrip=True, rstrip=True, normalized=False),
                        AddedToken("[SEP]", special=False, rstrip=True, normalized=True)])
    data = json.loads(tok.to_str())
    if kind == "qwen2":
        # merges as "a b" strings, as the reference's loader reads them
        data["model"]["merges"] = [" ".join(m) if isinstance(m, list) else m for m in data["model"]["merges"]]
    return data


def main():
    rng = random.Random(20261202)
    corpus = [text(rng, rng.randint(20, 120)) for _ in range(4000)]
    case_rng = random.Random(7)
    cases = edge_cases() + [text(case_rng, case_rng.randint(1, 40)) for _ in range(220)]
    golden = {"cases": cases, "expect": {}}
    for kind in ("qwen2", "llama3", "gpt2"):
        data = train(kind, corpus)
        path = os.path.join(HERE, f"tokenizer_{kind}.json")
        with open(path, "w", encoding="utf-8") as f:
            json.dump(data, f, ensure_ascii=False, separators=(",", ":"))
        tok = Tokenizer.from_file(path)
        plain = [tok.encode(c, add_special_tokens=False).ids for c in cases]
        with_post = [tok.encode(c, add_special_tokens=True).ids for c in cases]
        tok.encode_special_tokens = True
        as_text = [tok.encode(c, add_special_tokens=False).ids for c in cases]
        tok.encode_special_tokens = False
        # stored compactly: the post-processor adds a fixed prefix; the other
        # three are kept only where they differ from ids / the case text
        prefix = with_post[0][:len(with_post[0]) - len(plain[0])]
        assert all(w == prefix + p for w, p in zip(with_post, plain))
        dec = [tok.decode(ids, skip_special_tokens=False) for ids in plain]
        dec_skip = [tok.decode(ids, skip_special_tokens=True) for ids in plain]
        golden["expect"][kind] = {
            "ids": plain,
            "add_special_prefix": prefix,
            "ids_special_as_text": {str(i): a for i, (a, p) in enumerate(zip(as_text, plain)) if a != p},
            "decoded": {str(i): d for i, d in enumerate(dec) if d != cases[i]},
            "decoded_skip_special": {str(i): d for i, d in enumerate(dec_skip) if d != dec[i]},
        }
    with open(os.path.join(HERE, "tokenizer_cases.json"), "w", encoding="utf-8") as f:
        json.dump(golden, f, ensure_ascii=False, separators=(",", ":"))


if __name__ == "__main__":
    main()
