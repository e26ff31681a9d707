"""Writes tests/golden/bridge_symbols.json: the C functions the reference's
native bridge declares (inference/native/bridge.hpp) and the names its Rust
crate resolves when it loads that library (Kitchen::load,
inference/src/native.rs:1299-1354).  Reads the reference tree as text only.

    python tests/golden/make_bridge_symbols.py /path/to/reference
"""
import json
import os
import re
import sys


def main(ref: str) -> None:
    hpp = open(os.path.join(ref, "inference/native/bridge.hpp")).read()
    body = hpp[hpp.index('extern "C" {'):]
    declared = sorted(set(re.findall(r"\b(imagine_[A-Za-z0-9_]+)\s*\(", body)))
    rs = open(os.path.join(ref, "inference/src/native.rs")).read()
    load = rs[rs.index("let loaded = (|| unsafe {"):]
    load = load[:load.index("})();")]
    resolved = re.findall(r'symbol\(handle,\s*c"(imagine_[A-Za-z0-9_]+)"\)', load)
    out = {"source": "inference/native/bridge.hpp (extern \"C\" block); "
                     "inference/src/native.rs:1299-1354 (Kitchen::load)",
           "bridge_hpp": declared, "kitchen_load": resolved}
    path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "bridge_symbols.json")
    with open(path, "w") as f:
        json.dump(out, f, indent=1)
    print(f"{len(declared)} declared, {len(resolved)} resolved -> {path}")


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else "/root/reference")
