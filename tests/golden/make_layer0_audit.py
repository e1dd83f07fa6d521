"""Write the static operation audit of the reference's Layer-0 preset.

    python tests/golden/make_layer0_audit.py

Runs ``llama3fhe.application.runner.main(['--audit-only'], layer0_preset=True)``
(``application/runner.py:188-200``, ``graph.operation_audit`` at
``graph.py:348-542``) from the installed reference tree with this repository's
``easyfhe`` as its backend (the audit calls ``bs.requirements`` for the
bootstrap rotations), and writes ``layer0_audit.json`` beside this script:
the op counts per stage and the rotation-key count.  ``tests/test_reference_layer.py``
re-runs the audit and compares.
"""

from __future__ import annotations

import contextlib
import io
import json
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent.parent / "easyfhe-llama3-8b_b200"))


def audit_payload() -> dict:
    import llama3_layer

    llama3_layer.import_reference()
    from llama3fhe.application import runner

    buf = io.StringIO()
    with contextlib.redirect_stdout(buf):
        runner.main(["--audit-only"], layer0_preset=True)
    text = buf.getvalue()
    payload = json.loads(text[text.index("{"):])
    return {"rotation_key_count": payload["rotation_key_count"],
            "canonical_cipher_count": payload["canonical_cipher_count"],
            "polynomial_degrees": payload["polynomial_degrees"],
            "audit": payload["audit"]}


if __name__ == "__main__":
    out = HERE / "layer0_audit.json"
    out.write_text(json.dumps(audit_payload(), indent=1, sort_keys=True) + "\n")
    print(f"wrote {out}")
