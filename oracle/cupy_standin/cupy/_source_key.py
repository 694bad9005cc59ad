"""Key of one compiled kernel module: the source text and the compile options, as CuPy
keys its own kernel cache (TEST INFRASTRUCTURE ONLY)."""
import hashlib


def source_key(code, options=()):
    h = hashlib.sha256()
    h.update(code.encode("utf-8"))
    for opt in options:
        h.update(b"\0")
        h.update(str(opt).encode("utf-8"))
    return h.hexdigest()[:32]
