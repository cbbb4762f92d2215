"""Every `uses:` of a GitHub workflow names a third-party action by a full 40-hex commit SHA
(a tag can be moved to other code after review).  Exit 1 and list the offending lines otherwise.

    python ci/check_action_pins.py [workflow dir]
"""
import os
import re
import sys

USES = re.compile(r"^\s*-?\s*uses:\s*([^\s#]+)")
PINNED = re.compile(r"^[\w.-]+/[\w./-]+@[0-9a-f]{40}$")


def check(root):
    bad = []
    for name in sorted(os.listdir(root)):
        if not name.endswith((".yml", ".yaml")):
            continue
        with open(os.path.join(root, name), encoding="utf-8") as f:
            for n, line in enumerate(f, 1):
                m = USES.match(line)
                if m and not m.group(1).startswith("./") and not PINNED.match(m.group(1)):
                    bad.append(f"{name}:{n}: {m.group(1)}")
    return bad


def main(argv=None):
    argv = sys.argv[1:] if argv is None else argv
    root = argv[0] if argv else os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))),
                                             ".github", "workflows")
    bad = check(root)
    for b in bad:
        print(f"unpinned action: {b}")
    return 1 if bad else 0


if __name__ == "__main__":
    sys.exit(main())
