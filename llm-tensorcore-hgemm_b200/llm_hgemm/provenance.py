"""Source fingerprint binding a dispatch policy file to the code it was tuned
on (reference llm_hgemm/provenance.py:7-22). Called off the hot path only.

The fingerprint covers the kernel and host sources, the C-ABI header and this
package's Python files; built shared objects are excluded so that a rebuild
of the same sources keeps the fingerprint.
"""

from hashlib import sha256
from pathlib import Path

PKG_ROOT = Path(__file__).resolve().parents[1]
REPO_ROOT = PKG_ROOT.parent
_SUFFIXES = {".py", ".cu", ".cuh", ".cpp", ".h"}


def file_sha256(path) -> str:
    return sha256(Path(path).read_bytes()).hexdigest()


def _sources() -> list[tuple[str, Path]]:
    found = []
    for folder in (PKG_ROOT / "csrc", PKG_ROOT / "llm_hgemm", REPO_ROOT / "include"):
        for p in folder.rglob("*"):
            if p.is_file() and p.suffix in _SUFFIXES and "__pycache__" not in p.parts:
                found.append((str(p.relative_to(REPO_ROOT)), p))
    build = PKG_ROOT / "build.py"
    if build.exists():
        found.append((str(build.relative_to(REPO_ROOT)), build))
    return sorted(found)


def code_fingerprint() -> str:
    digest = sha256()
    for rel, path in _sources():
        digest.update(rel.encode())
        digest.update(path.read_bytes())
    return digest.hexdigest()
