# SPDX-License-Identifier: Apache-2.0
"""Extract the reference's committed query-session golden records.

Reads ``data/query_session/correctness.json`` of the GSA reference checkout
(the argument, else the ``GSA_REFERENCE`` environment variable) and writes ``query_session_correctness.json``
beside this script: for each of the 94 calls of the reference test
``tests/check_queries.py`` its op, label, sizes, radius, K, the SHA-256 of
the int32 output rows (radius calls) and the session statistics after the
call.  The reference checkout is only needed to regenerate the fixture; the
tests read the committed fixture.

Usage: python tests/golden/make_golden.py [REFERENCE_ROOT]
"""

import json
import os
import sys
from pathlib import Path

if len(sys.argv) > 1:
    root = Path(sys.argv[1])
elif os.environ.get("GSA_REFERENCE"):
    root = Path(os.environ["GSA_REFERENCE"])
else:
    sys.exit("usage: make_golden.py REFERENCE_ROOT (or set GSA_REFERENCE)")
src = json.loads((root / "data/query_session/correctness.json").read_text())
keep = ("op", "label", "n", "q", "r", "k", "ids_sha256", "stats")
records = [{k: r[k] for k in keep if k in r} for r in src["records"]]
assert len(records) == src["calls"] == 94
out = Path(__file__).with_name("query_session_correctness.json")
out.write_text(
    json.dumps(
        {
            "source": "GSA data/query_session/correctness.json (reference run of tests/check_queries.py)",
            "seed": 20261111,
            "calls": len(records),
            "records": records,
        },
        indent=1,
    )
    + "\n"
)
print(f"wrote {out} ({len(records)} records)")
