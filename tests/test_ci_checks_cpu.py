"""Repository checks run by CI: pinned workflow actions, first-party product code."""
import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(ROOT, "ci"))


def test_action_pins(tmp_path):
    import check_action_pins as C
    (tmp_path / "a.yml").write_text("steps:\n  - uses: actions/checkout@11bd71901bbe5b1630ceea73d27597364c9af683\n"
                                    "  - uses: actions/setup-python@v5\n  - uses: ./local-action\n")
    assert C.check(str(tmp_path)) == ["a.yml:3: actions/setup-python@v5"]
    assert C.main([os.path.join(ROOT, ".github", "workflows")]) == 0


def test_product_is_first_party():
    import check_first_party as C
    assert C.check() == []
