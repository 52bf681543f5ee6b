"""Generates unicode_tables.inc, the character data of the host tokenizer
(tokenizer.cpp).

HF tokenizer.json files are written for the `tokenizers` library, and the
tokenizer here must split and normalise text exactly as that library does.
Its regex engine and its NFC normaliser carry different Unicode versions (the
regex classes follow Unicode 16, the same tables the reference ships in
src/tokenizer/unicode_tables.h; the normaliser follows an older release).  So
every table below is read off the library's own behaviour, code point by code
point, rather than off Python's `unicodedata`:

  * \\p{L}, \\p{N}, \\s   -- a Split pre-tokenizer with the class as its
                           pattern, run over every code point;
  * word characters      -- the code points beside which the library drops
                           a match of a single_word added token (either side);
  * full canonical        -- NFD of each code point;
    decompositions
  * combining classes     -- the order NFD puts a mark in next to a mark of
                           each known class;
  * primary composites    -- the code points whose decomposition NFC puts
                           back together (pairs from Python's first-level
                           mappings, kept only where the library agrees).

Usage: python gen_unicode_tables.py  (writes unicode_tables.inc beside it);
tests/test_tokenizer.py regenerates the text with build_tables() and compares.
"""
import os
import sys
import unicodedata

from tokenizers import AddedToken, Regex, Tokenizer, models, normalizers, pre_tokenizers

HERE = os.path.dirname(os.path.abspath(__file__))
SEP = "\x00"  # a starter with no decomposition that nothing composes with
ALL = [c for c in range(1, 0x110000) if not (0xD800 <= c <= 0xDFFF)]


def ranges(members):
    out, start, prev = [], None, None
    for c in sorted(members):
        if start is None:
            start = c
        elif c != prev + 1:
            out.append((start, prev))
            start = c
        prev = c
    if start is not None:
        out.append((start, prev))
    return out


def class_members(cls):
    """Code points the library's regex engine puts in `cls`."""
    split = pre_tokenizers.Split(Regex(cls), behavior="removed")
    outside = set()
    for i in range(0, len(ALL), 50000):
        block = "".join(chr(c) for c in ALL[i:i + 50000])
        for piece, _ in split.pre_tokenize_str(block):
            outside.update(ord(ch) for ch in piece)
    return set(ALL) - outside


def word_members():
    """Code points next to which the library skips a single_word added token's
    match (checked on both sides; they agree)."""
    alphabet = sorted(pre_tokenizers.ByteLevel.alphabet())
    tok = Tokenizer(models.BPE(vocab={ch: i for i, ch in enumerate(alphabet)}, merges=[]))
    tok.pre_tokenizer = pre_tokenizers.ByteLevel(add_prefix_space=False, use_regex=False)
    tok.add_tokens([AddedToken("qqzz", single_word=True, normalized=False, special=False)])
    tid = tok.token_to_id("qqzz")
    left = tok.encode_batch([chr(c) + "qqzz" for c in ALL], add_special_tokens=False)
    right = tok.encode_batch(["qqzz" + chr(c) for c in ALL], add_special_tokens=False)
    wl = {c for c, e in zip(ALL, left) if tid not in e.ids}
    wr = {c for c, e in zip(ALL, right) if tid not in e.ids}
    assert wl == wr
    return wl


def batch(norm, strings, chunk=100000):
    out = []
    for i in range(0, len(strings), chunk):
        part = strings[i:i + chunk]
        res = norm.normalize_str(SEP.join(part)).split(SEP)
        assert len(res) == len(part)
        out.extend(res)
    return out


def build_tables():
    """The text of unicode_tables.inc and a one-line summary."""
    letters, numbers, spaces = class_members(r"\p{L}"), class_members(r"\p{N}"), class_members(r"\s")
    words = word_members()
    nfd, nfc = normalizers.NFD(), normalizers.NFC()

    # full canonical decompositions (Hangul syllables are algorithmic and left out)
    d_all = batch(nfd, [chr(c) for c in ALL])
    decomp = {}
    for c, d in zip(ALL, d_all):
        if d != chr(c) and not (0xAC00 <= c <= 0xD7A3):
            decomp[c] = [ord(x) for x in d]
    assert [ord(x) for x in nfd.normalize_str("각")] == [0x1100, 0x1161, 0x11A8]

    # combining classes: a mark m of class k and a probe p of class v are
    # swapped by NFD("a" p m) iff k < v, and by NFD("a" m p) iff v < k.
    cands = [c for c in ALL if unicodedata.combining(chr(c)) and c not in decomp]
    # one probe per class: the lowest code point of that class that the
    # library treats as a non-starter (it swaps with U+0345, class 240, or for
    # class 240 itself with U+0300, class 230)
    def non_starter(p, v):
        if v == 240:
            return nfd.normalize_str("a\u0345\u0300") == "a\u0300\u0345" and p == 0x345
        return nfd.normalize_str("a\u0345" + chr(p)) == "a" + chr(p) + "\u0345"
    probes = {}
    for c in sorted(ALL):
        v = unicodedata.combining(chr(c))
        if v and v not in probes and c not in decomp and non_starter(c, v):
            probes[v] = c
    vals = sorted(probes)
    ccc = {}
    for v in vals:
        p = chr(probes[v])
        before = batch(nfd, ["a" + p + chr(c) for c in cands])   # swapped: k < v
        after = batch(nfd, ["a" + chr(c) + p for c in cands])    # swapped: v < k
        for c, b, a in zip(cands, before, after):
            lt = b != "a" + p + chr(c)
            gt = a != "a" + chr(c) + p
            ccc.setdefault(c, []).append((v, lt, gt))
    cls = {}
    for c, obs in ccc.items():
        k = None
        # the library's class for c is the probe class with neither swap
        # (c is a non-starter only if some probe swaps with it)
        if any(lt or gt for _, lt, gt in obs):
            eq = [v for v, lt, gt in obs if not lt and not gt]
            assert len(eq) == 1, (hex(c), eq)
            k = eq[0]
        if k:
            cls[c] = k
    # no code point outside the candidates is a non-starter in the library
    full = dict(zip(ALL, d_all))
    others = [c for c in ALL if c not in cls and ord(full[c][0]) not in cls]
    swapped = batch(nfd, ["a\u0345" + chr(c) for c in others])
    assert all(s == "a\u0345" + full[c] for c, s in zip(others, swapped))

    # primary composites: first-level pairs whose NFD the library recomposes
    compose = []
    for c in ALL:
        if c not in decomp:
            continue
        m = unicodedata.decomposition(chr(c))
        if not m or m.startswith("<"):
            continue
        parts = [int(x, 16) for x in m.split()]
        if len(parts) != 2:
            continue
        if nfc.normalize_str("".join(chr(x) for x in decomp[c])) == chr(c):
            compose.append((parts[0], parts[1], c))
    compose.sort()

    ccc_ranges = []
    for c in sorted(cls):
        if ccc_ranges and ccc_ranges[-1][1] == c - 1 and ccc_ranges[-1][2] == cls[c]:
            ccc_ranges[-1][1] = c
        else:
            ccc_ranges.append([c, c, cls[c]])

    out = []
    out.append("// Generated by gen_unicode_tables.py from the HF `tokenizers` library's own\n"
               "// regex classes and NFC normaliser; do not edit.\n")

    def emit_ranges(name, rs):
        out.append(f"static const CpRange {name}[] = {{\n")
        for a, b in rs:
            out.append(f"    {{0x{a:X}, 0x{b:X}}},\n")
        out.append("};\n")

    emit_ranges("kLetterRanges", ranges(letters))
    emit_ranges("kNumberRanges", ranges(numbers))
    emit_ranges("kSpaceRanges", ranges(spaces))
    emit_ranges("kWordRanges", ranges(words))
    out.append("static const CccRange kCccRanges[] = {\n")
    for a, b, v in ccc_ranges:
        out.append(f"    {{0x{a:X}, 0x{b:X}, {v}}},\n")
    out.append("};\n")
    data, entries = [], []
    for c in sorted(decomp):
        entries.append((c, len(data), len(decomp[c])))
        data.extend(decomp[c])
    out.append("static const uint32_t kDecompData[] = {\n")
    for i in range(0, len(data), 8):
        out.append("    " + ", ".join(f"0x{x:X}" for x in data[i:i + 8]) + ",\n")
    out.append("};\n")
    out.append("static const DecompEntry kDecomp[] = {\n")
    for c, off, n in entries:
        out.append(f"    {{0x{c:X}, {off}, {n}}},\n")
    out.append("};\n")
    out.append("static const ComposePair kCompose[] = {\n")
    for a, b, c in compose:
        out.append(f"    {{0x{a:X}, 0x{b:X}, 0x{c:X}}},\n")
    out.append("};\n")
    summary = (f"{len(ranges(letters))} letter, {len(ranges(numbers))} number, "
               f"{len(ranges(spaces))} space, {len(ranges(words))} word ranges; {len(ccc_ranges)} class ranges; "
               f"{len(entries)} decompositions; {len(compose)} composites")
    return "".join(out), summary


def main():
    text, summary = build_tables()
    path = os.path.join(HERE, "unicode_tables.inc")
    with open(path, "w") as f:
        f.write(text)
    print(f"{path}: {summary}", file=sys.stderr)


if __name__ == "__main__":
    main()
