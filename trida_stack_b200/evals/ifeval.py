"""IFEval instruction checkers and scoring, written for this package (no third-party evaluator).

The reference runs Google's IFEval evaluator (vendored in ``inference/zoro-1/ifeval_lib``, driven
by ``eval_ifeval.py``).  This module checks the same 25 instruction ids with the same keyword
arguments and the same prompt-level / instruction-level, strict / loose scores:

* strict: the response (with any ``<think>`` block removed) is checked as is;
* loose: an instruction also counts as followed if it holds for one of the variants made by
  dropping the first line, the last line or both, each with and without the ``*`` characters.

Two checks rely on natural-language tooling the image does not ship: sentences are split with a
punctuation rule (``. ! ?`` followed by space and an upper-case / digit / quote start, common
abbreviations excepted) and the response language is identified from its script (Cyrillic,
Arabic, Devanagari, Hangul, Thai, Bengali, ...) and, for Latin-script languages, from function-word
frequencies.  Results can therefore differ slightly from runs with nltk / langdetect.
"""
import json
import re
import string
import unicodedata

# ------------------------------------------------------------------------------------ text tools
_ABBREV = {"mr", "mrs", "ms", "dr", "prof", "sr", "jr", "st", "vs", "etc", "e.g", "i.e", "inc", "ltd", "co",
           "u.s", "u.k", "no", "fig", "approx", "dept", "est", "jan", "feb", "mar", "apr", "jun", "jul", "aug",
           "sep", "sept", "oct", "nov", "dec"}


def split_sentences(text):
    text = text.strip()
    if not text:
        return []
    out, start = [], 0
    for m in re.finditer(r"[.!?]+[\"')\]]*\s+", text):
        end = m.end()
        head = text[start:m.start()].rstrip()
        last = head.split()[-1].lower().rstrip(".") if head.split() else ""
        nxt = text[end:end + 1]
        if last in _ABBREV or (len(last) == 1 and last.isalpha() and m.group(0).startswith(".")):
            continue
        if nxt and not (nxt.isupper() or nxt.isdigit() or nxt in "\"'(["):
            continue
        out.append(text[start:end].strip())
        start = end
    if start < len(text):
        out.append(text[start:].strip())
    return [s for s in out if s]


def count_words(text):
    return len(re.findall(r"\b\w+(?:['’]\w+)?\b", text))


_SCRIPTS = [  # (language code, first and last code point of its script block)
    ("ru", 0x0400, 0x04FF), ("ar", 0x0600, 0x06FF), ("hi", 0x0900, 0x097F), ("bn", 0x0980, 0x09FF),
    ("pa", 0x0A00, 0x0A7F), ("gu", 0x0A80, 0x0AFF), ("ta", 0x0B80, 0x0BFF), ("te", 0x0C00, 0x0C7F),
    ("kn", 0x0C80, 0x0CFF), ("ml", 0x0D00, 0x0D7F), ("th", 0x0E00, 0x0E7F), ("ko", 0xAC00, 0xD7AF),
    ("ja", 0x3040, 0x30FF), ("zh", 0x4E00, 0x9FFF), ("el", 0x0370, 0x03FF), ("he", 0x0590, 0x05FF),
]
_STOP = {
    "en": "the and of to is in that it for you with was are this be on not as have",
    "es": "el la de que y en los se las por un una es con para no del",
    "fr": "le la les de et des est un une que en du pour pas dans qui",
    "de": "der die und das ist nicht den ein eine zu mit von sich des auf für",
    "it": "il di che la e per un una non sono del della gli le con",
    "pt": "o a de que e os as um uma não do da em para com por",
    "nl": "de het een en van is dat niet in op te zijn voor met",
    "fi": "ja on ei se että oli ovat mutta kun tai joka myös niin",
    "sv": "och att det som en är på av för med inte den till har",
    "vi": "và của là có không những được trong cho với một các người",
    "sw": "na ya wa kwa ni la za katika kama hii huo cha",
    "tr": "ve bir bu da de için ile ne çok daha olarak gibi",
}
_STOP = {k: set(v.split()) for k, v in _STOP.items()}


def detect_language(text):
    """ISO code of the dominant language (script first, then Latin function words)."""
    counts = {}
    letters = 0
    for ch in text:
        if not ch.isalpha():
            continue
        letters += 1
        cp = ord(ch)
        for code, lo, hi in _SCRIPTS:
            if lo <= cp <= hi:
                counts[code] = counts.get(code, 0) + 1
                break
    if letters == 0:
        return "unknown"
    if counts:
        code, n = max(counts.items(), key=lambda kv: kv[1])
        if n > 0.3 * letters:
            if code == "ar" and re.search(r"[پچژگ]", text):
                return "fa"
            if code == "ar" and re.search(r"[ٹڈڑں]", text):
                return "ur"
            if code == "hi" and re.search(r"[ळ]", text) and "आहे" in text:
                return "mr"
            if code == "ru" and re.search(r"[ъ]", text) and not re.search(r"[ыэё]", text):
                return "bg"
            return code
    words = re.findall(r"[^\W\d_]+", text.lower())
    best, score = "en", -1.0
    for code, stop in _STOP.items():
        s = sum(w in stop for w in words) / max(len(words), 1)
        if s > score:
            best, score = code, s
    return best


def _rel(n, target, relation):
    if relation == "less than":
        return n < target
    if relation == "at least":
        return n >= target
    raise ValueError(f"unknown relation {relation!r}")


# ------------------------------------------------------------------------------------ checkers
def _keywords_existence(r, keywords, **_):
    return all(re.search(re.escape(k), r, re.IGNORECASE) for k in keywords)


def _keywords_frequency(r, keyword, frequency, relation, **_):
    return _rel(len(re.findall(re.escape(keyword), r, re.IGNORECASE)), frequency, relation)


def _forbidden(r, forbidden_words, **_):
    return not any(re.search(r"\b" + re.escape(w) + r"\b", r, re.IGNORECASE) for w in forbidden_words)


def _letter_frequency(r, letter, let_frequency, let_relation, **_):
    return _rel(r.lower().count(letter.lower()), let_frequency, let_relation)


def _language(r, language, **_):
    return detect_language(r) == language


def _num_sentences(r, num_sentences, relation, **_):
    return _rel(len(split_sentences(r)), num_sentences, relation)


def _num_paragraphs(r, num_paragraphs, **_):
    parts = re.split(r"\s?\*\*\*\s?", r)
    n = len(parts)
    for i, p in enumerate(parts):
        if not p.strip():
            if i == 0 or i == len(parts) - 1:
                n -= 1
            else:
                return False
    return n == num_paragraphs


def _num_words(r, num_words, relation, **_):
    return _rel(count_words(r), num_words, relation)


def _nth_paragraph_first_word(r, num_paragraphs, nth_paragraph, first_word, **_):
    paras = [p for p in re.split(r"\n\n", r) if p.strip()]
    if len(paras) != num_paragraphs or nth_paragraph > len(paras):
        return False
    p = paras[nth_paragraph - 1].strip()
    word = ""
    for tok in p.split():
        word = tok.lstrip(string.punctuation + "“‘\"'").rstrip(string.punctuation + "”’\"'")
        if word:
            break
    return word.lower() == first_word.lower()


def _placeholders(r, num_placeholders, **_):
    return len(re.findall(r"\[.*?\]", r)) >= num_placeholders


def _postscript(r, postscript_marker, **_):
    m = postscript_marker.strip().lower()
    if m == "p.p.s":
        pat = r"\s*p\.\s?p\.\s?s.*$"
    elif m == "p.s.":
        pat = r"\s*p\.\s?s\..*$"
    else:
        pat = r"\s*" + re.escape(m) + r".*$"
    return re.search(pat, r.lower(), re.MULTILINE) is not None


def _bullets(r, num_bullets, **_):
    n = len(re.findall(r"^\s*\*[^\*].*$", r, re.MULTILINE)) + len(re.findall(r"^\s*-.*$", r, re.MULTILINE))
    return n == num_bullets


def _constrained(r, **_):
    return any(o in r.strip() for o in ("My answer is yes.", "My answer is no.", "My answer is maybe."))


def _highlights(r, num_highlights, **_):
    n = sum(1 for h in re.findall(r"\*[^\n\*]*\*", r) if h.strip("*").strip())
    n += sum(1 for h in re.findall(r"\*\*[^\n\*]*\*\*", r) if h.removeprefix("**").removesuffix("**").strip())
    return n >= num_highlights


def _sections(r, section_spliter, num_sections, **_):
    parts = re.split(r"\s?" + re.escape(section_spliter) + r"\s?\d+\s?", r)
    return len(parts) - 1 >= num_sections


def _json(r, **_):
    v = r.strip()
    for pre in ("```json", "```Json", "```JSON", "```"):
        v = v.removeprefix(pre)
    v = v.removesuffix("```").strip()
    try:
        json.loads(v)
    except ValueError:
        return False
    return True


def _title(r, **_):
    return any(t.lstrip("<").rstrip(">").strip() for t in re.findall(r"<<[^\n]+>>", r))


def _two_responses(r, **_):
    parts = r.split("******")
    valid = [p.strip() for p in parts if p.strip()]
    if len(parts) - len(valid) > 2 or len(valid) != 2:
        return False
    return valid[0] != valid[1]


def _repeat_prompt(r, prompt_to_repeat, **_):
    return r.strip().lower().startswith(prompt_to_repeat.strip().lower())


def _end_checker(r, end_phrase, **_):
    return r.strip().strip("\"").lower().endswith(end_phrase.strip().lower())


def _capital_words(r, capital_frequency, capital_relation, **_):
    words = re.findall(r"\b\w+\b", r)
    return _rel(sum(1 for w in words if w.isupper()), capital_frequency, capital_relation)


def _english_capital(r, **_):
    return r.isupper() and detect_language(r) == "en"


def _english_lowercase(r, **_):
    return r.islower() and detect_language(r) == "en"


def _no_comma(r, **_):
    return "," not in r


def _quotation(r, **_):
    v = r.strip()
    return len(v) > 1 and v[0] == '"' and v[-1] == '"'


CHECKERS = {
    "keywords:existence": _keywords_existence,
    "keywords:frequency": _keywords_frequency,
    "keywords:forbidden_words": _forbidden,
    "keywords:letter_frequency": _letter_frequency,
    "language:response_language": _language,
    "length_constraints:number_sentences": _num_sentences,
    "length_constraints:number_paragraphs": _num_paragraphs,
    "length_constraints:number_words": _num_words,
    "length_constraints:nth_paragraph_first_word": _nth_paragraph_first_word,
    "detectable_content:number_placeholders": _placeholders,
    "detectable_content:postscript": _postscript,
    "detectable_format:number_bullet_lists": _bullets,
    "detectable_format:constrained_response": _constrained,
    "detectable_format:number_highlighted_sections": _highlights,
    "detectable_format:multiple_sections": _sections,
    "detectable_format:json_format": _json,
    "detectable_format:title": _title,
    "combination:two_responses": _two_responses,
    "combination:repeat_prompt": _repeat_prompt,
    "startend:end_checker": _end_checker,
    "change_case:capital_word_frequency": _capital_words,
    "change_case:english_capital": _english_capital,
    "change_case:english_lowercase": _english_lowercase,
    "punctuation:no_comma": _no_comma,
    "startend:quotation": _quotation,
}


def strip_thinking(text):
    return re.sub(r"^.*</think>\s*", "", text or "", count=1, flags=re.DOTALL)


def _loose_variants(r):
    lines = r.split("\n")
    base = [r, "\n".join(lines[1:]).strip(), "\n".join(lines[:-1]).strip(), "\n".join(lines[1:-1]).strip()]
    return base + [v.replace("*", "") for v in base]


def follows(instruction_id, response, kwargs, loose=False):
    fn = CHECKERS[instruction_id]
    kw = {k: v for k, v in (kwargs or {}).items() if v is not None}
    if not loose:
        return bool(response.strip()) and bool(fn(response, **kw))
    return any(v.strip() and fn(v, **kw) for v in _loose_variants(response))


def score_example(example, response):
    """(strict list, loose list) of per-instruction results for one IFEval record."""
    r = strip_thinking(response)
    ids, kws = example["instruction_id_list"], example["kwargs"]
    return ([follows(i, r, kw) for i, kw in zip(ids, kws)], [follows(i, r, kw, loose=True) for i, kw in zip(ids, kws)])


def aggregate(results):
    """Prompt- and instruction-level accuracies (%) from a list of (strict, loose) lists."""
    def acc(sel):
        prompts = [all(x) for x in sel]
        inst = [v for x in sel for v in x]
        return (round(100 * sum(prompts) / max(len(prompts), 1), 2), round(100 * sum(inst) / max(len(inst), 1), 2))
    ps, is_ = acc([s for s, _ in results])
    pl, il = acc([l for _, l in results])
    return {"prompt_strict": ps, "instruction_strict": is_, "prompt_loose": pl, "instruction_loose": il,
            "n": len(results)}


def normalize(text):
    return unicodedata.normalize("NFKC", text)
