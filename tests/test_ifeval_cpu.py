"""IFEval instruction checks (own implementation): strict / loose semantics on hand-made cases."""
from trida_stack_b200.evals import ifeval as F


def ok(iid, text, loose=False, **kw):
    return F.follows(iid, text, kw, loose=loose)


def test_keyword_and_length_checks():
    assert ok("keywords:existence", "Blue whales are big.", keywords=["whale", "big"])
    assert not ok("keywords:existence", "Blue whales.", keywords=["whale", "big"])
    assert ok("keywords:frequency", "a cat, a cat, a cat", keyword="cat", frequency=3, relation="at least")
    assert not ok("keywords:frequency", "cat cat cat", keyword="cat", frequency=3, relation="less than")
    assert ok("keywords:forbidden_words", "scatter plots", forbidden_words=["cat"])      # whole words only
    assert not ok("keywords:forbidden_words", "the Cat sat", forbidden_words=["cat"])
    assert ok("keywords:letter_frequency", "banana", letter="a", let_frequency=3, let_relation="at least")
    assert ok("length_constraints:number_words", "one two three", num_words=4, relation="less than")
    assert ok("length_constraints:number_sentences", "Hi there. Dr. Smith came! Why? Yes.", num_sentences=4,
              relation="at least")
    assert not ok("length_constraints:number_sentences", "Hi there. Dr. Smith came! Why? Yes.", num_sentences=4,
                  relation="less than")
    assert ok("length_constraints:number_paragraphs", "a\n***\nb\n***\nc", num_paragraphs=3)
    assert not ok("length_constraints:number_paragraphs", "a\n***\n\n***\nc", num_paragraphs=3)
    assert ok("length_constraints:nth_paragraph_first_word", "Intro text.\n\n\"Second\" para.", num_paragraphs=2,
              nth_paragraph=2, first_word="second")


def test_format_checks():
    assert ok("detectable_format:number_bullet_lists", "* a\n* b\n- c", num_bullets=3)
    assert ok("detectable_format:number_highlighted_sections", "*one* and **two**", num_highlights=2)
    assert ok("detectable_format:multiple_sections", "SECTION 1\nx\nSECTION 2\ny", section_spliter="SECTION",
              num_sections=2)
    assert ok("detectable_format:json_format", '```json\n{"a": 1}\n```')
    assert not ok("detectable_format:json_format", "{a: 1}")
    assert ok("detectable_format:title", "<<My Title>>\ntext")
    assert ok("detectable_format:constrained_response", "Thinking... My answer is no.")
    assert ok("detectable_content:number_placeholders", "Dear [name], at [address]", num_placeholders=2)
    assert ok("detectable_content:postscript", "Body\nP.S. see you", postscript_marker="P.S.")
    assert ok("combination:two_responses", "first\n******\nsecond")
    assert not ok("combination:two_responses", "same\n******\nsame")
    assert ok("combination:repeat_prompt", "Write a poem. Here it is", prompt_to_repeat="write a poem.")
    assert ok("startend:end_checker", "... Any other questions?", end_phrase="Any other questions?")
    assert ok("startend:quotation", '"quoted answer"')
    assert ok("punctuation:no_comma", "no commas here")
    assert ok("change_case:english_lowercase", "all lowercase english text is here and it is fine")
    assert ok("change_case:english_capital", "THIS IS ALL CAPS AND IT IS THE ANSWER")
    assert ok("change_case:capital_word_frequency", "THE END is NEAR", capital_frequency=3,
              capital_relation="at least")


def test_language_detection_and_loose_variants():
    assert F.detect_language("Это простой ответ на русском языке.") == "ru"
    assert F.detect_language("यह हिंदी में लिखा गया उत्तर है।") == "hi"
    assert F.detect_language("Esta es una respuesta escrita en español para la prueba.") == "es"
    assert F.detect_language("This is an answer that is written in English for the test.") == "en"
    # a preamble line breaks strict quotation but loose drops the first line
    text = 'Sure, here you go:\n"quoted answer"'
    assert not ok("startend:quotation", text) and ok("startend:quotation", text, loose=True)
    ex = {"instruction_id_list": ["punctuation:no_comma", "startend:quotation"], "kwargs": [{}, {}]}
    strict, loose = F.score_example(ex, "<think>a, b</think>" + text)
    agg = F.aggregate([(strict, loose)])
    assert strict == [False, False] or strict == [True, False]
    assert agg["prompt_loose"] == 100.0 and agg["n"] == 1
