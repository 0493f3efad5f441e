"""Copy the reference's triangle-multiplication golden bundles into tests/golden/.

The reference keeps four frozen bundles for the outgoing triangle update
(test/fixtures/openfold-triangle-small, test/fixtures/alphafold-single-sequence/
{short-9,model1-reference-59}, test/fixtures/alphafold-a3m/model1-reference-59).
Each bundle is a manifest.json plus raw little-endian float32 tensors in the
format read by src/reference/node.ts:13-42 (manifest layout src/reference/bundle.ts:1-20).

The GPU box has no copy of the reference tree, so the bundles travel with this
repository. The tensors are copied byte for byte; nothing is regenerated. The
AlphaFold parameters inside the three AlphaFold bundles are DeepMind's, under
the CC BY 4.0 parameters licence (see tests/golden/README.md).

Run once, in a container that holds the reference checkout:

    python tests/golden/make_golden.py /path/to/reference
"""
from __future__ import annotations

import hashlib
import json
import shutil
import sys
from pathlib import Path

BUNDLES = {
    "openfold-triangle-small": "test/fixtures/openfold-triangle-small",
    "af2-short-9": "test/fixtures/alphafold-single-sequence/short-9",
    "af2-single-59": "test/fixtures/alphafold-single-sequence/model1-reference-59",
    "af2-a3m-59": "test/fixtures/alphafold-a3m/model1-reference-59",
}


def main(reference: Path) -> None:
    here = Path(__file__).resolve().parent
    digests = {}
    for name, rel in BUNDLES.items():
        src = reference / rel
        dst = here / name
        dst.mkdir(exist_ok=True)
        manifest = json.loads((src / "manifest.json").read_text())
        shutil.copyfile(src / "manifest.json", dst / "manifest.json")
        for record in manifest["tensors"].values():
            shutil.copyfile(src / record["file"], dst / record["file"])
            digests[f"{name}/{record['file']}"] = hashlib.sha256(
                (dst / record["file"]).read_bytes()).hexdigest()
    (here / "SHA256SUMS.json").write_text(json.dumps(digests, indent=1, sort_keys=True) + "\n")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: python tests/golden/make_golden.py <path of the reference checkout>")
    main(Path(sys.argv[1]))
