"""libimagine_kitchen_w8a8.so as a whole bridge library: it exports every
function the reference's bridge declares (inference/native/bridge.hpp), a
loader that resolves names the way the crate's Kitchen::load does
(inference/src/native.rs:1299-1354: dlsym in order, fail on the first
missing one) succeeds, and the functions it does not implement are passed
through to the library named by IMAGINE_KITCHEN_FALLBACK_LIBRARY (here a
stand-in compiled by the test), or fail with the bridge's RuntimeError code
and a message when there is none.  The name lists come from
tests/golden/bridge_symbols.json (tests/golden/make_bridge_symbols.py)."""
import ctypes
import json
import os
import subprocess
import sys
import textwrap

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
SHIM = os.path.join(ROOT, "imagine_b200", "libimagine_kitchen_w8a8.so")
NAMES = json.load(open(os.path.join(ROOT, "tests", "golden", "bridge_symbols.json")))


def _ensure_built():
    if not os.path.exists(SHIM):
        from imagine_b200 import build as B

        B.build()
        B.build_shim()


def test_fixture_lists_the_bridge():
    assert len(NAMES["kitchen_load"]) == 52
    assert set(NAMES["kitchen_load"]) <= set(NAMES["bridge_hpp"])
    for name in ("imagine_kitchen_call", "imagine_fp8_scaled_mm", "imagine_aten_boxed"):
        assert name in NAMES["kitchen_load"]


def test_kitchen_load_resolves_every_symbol():
    """dlopen(RTLD_LOCAL) + dlsym of each name in Kitchen::load's order."""
    _ensure_built()
    lib = ctypes.CDLL(SHIM, mode=os.RTLD_LOCAL | os.RTLD_NOW)
    for name in NAMES["kitchen_load"]:
        assert getattr(lib, name, None) is not None, f"Missing native symbol: {name}"
    for name in NAMES["bridge_hpp"]:
        assert getattr(lib, name, None) is not None, f"bridge.hpp declares {name}"


FAKE = textwrap.dedent(r"""
    #include <stdint.h>
    #include <stddef.h>
    #include <string.h>
    static const char* err = "";
    static int freed = 0;
    const char* imagine_last_error(void) { return err; }
    int imagine_last_accelerator_code(void) { return 3; }
    int imagine_cuda_device_count(int64_t* n) { *n = 7; err = ""; return 0; }
    int imagine_cat(const void* const* t, size_t n, int64_t dim, void** out) {
      err = "fake bridge: cat refused"; return -20;
    }
    int imagine_kitchen_call(const char* name, const void* args, size_t n, int64_t* result) {
      if (strcmp(name, "adaln") == 0) { *result = 42; return 0; }
      err = "fake bridge: unknown kernel"; return -1;
    }
    uint64_t imagine_tensor_identity(const void* t) { return 99; }
    const char* imagine_last_metadata(void) { return "fake metadata"; }
    void imagine_event_free(void* e) { freed += 1; }
    int fake_freed(void) { return freed; }
""")

PROBE = textwrap.dedent(r"""
    import ctypes, json, sys
    lib = ctypes.CDLL(sys.argv[1], mode=ctypes.RTLD_LOCAL)
    lib.imagine_last_error.restype = ctypes.c_char_p
    lib.imagine_last_metadata.restype = ctypes.c_char_p
    lib.imagine_tensor_identity.restype = ctypes.c_uint64
    lib.imagine_tensor_identity.argtypes = [ctypes.c_void_p]
    out = {}
    n = ctypes.c_int64(-1)
    out["count_rc"] = lib.imagine_cuda_device_count(ctypes.byref(n))
    out["count"] = n.value
    out["cat_rc"] = lib.imagine_cat(None, 0, 0, None)
    out["cat_err"] = lib.imagine_last_error().decode()
    out["cat_accel"] = lib.imagine_last_accelerator_code()
    res = ctypes.c_int64(0)
    out["call_rc"] = lib.imagine_kitchen_call(b"adaln", None, 0, ctypes.byref(res))
    out["call_res"] = res.value
    out["identity"] = lib.imagine_tensor_identity(None)
    out["metadata"] = lib.imagine_last_metadata().decode()
    lib.imagine_event_free(None)
    print(json.dumps(out))
""")


def _probe(env_extra):
    env = {k: v for k, v in os.environ.items() if k != "IMAGINE_KITCHEN_FALLBACK_LIBRARY"}
    env.update(env_extra)
    r = subprocess.run([sys.executable, "-c", PROBE, SHIM], capture_output=True, text=True,
                       env=env, timeout=120)
    assert r.returncode == 0, r.stderr
    return json.loads(r.stdout.strip().splitlines()[-1])


def test_functions_forward_to_the_fallback_library(tmp_path):
    _ensure_built()
    src = tmp_path / "fake_bridge.c"
    src.write_text(FAKE)
    so = tmp_path / "libfake_bridge.so"
    subprocess.run(["gcc", "-shared", "-fPIC", "-O1", str(src), "-o", str(so)], check=True)
    out = _probe({"IMAGINE_KITCHEN_FALLBACK_LIBRARY": str(so)})
    assert out["count_rc"] == 0 and out["count"] == 7
    # a failing forwarded call keeps its code; its message and accelerator
    # code become this library's
    assert out["cat_rc"] == -20 and out["cat_err"] == "fake bridge: cat refused"
    assert out["cat_accel"] == 3
    # kernel names imagine_kitchen_call does not map go to the fallback's
    assert out["call_rc"] == 0 and out["call_res"] == 42
    assert out["identity"] == 99 and out["metadata"] == "fake metadata"


def test_functions_fail_without_a_fallback_library():
    _ensure_built()
    out = _probe({})
    assert out["count_rc"] == -1 and out["count"] == -1
    assert out["cat_rc"] == -1 and "IMAGINE_KITCHEN_FALLBACK_LIBRARY is not set" in out["cat_err"]
    assert out["call_rc"] == -1
    assert out["identity"] == 0 and out["metadata"] == ""


@pytest.mark.parametrize("name", ["imagine_cat", "imagine_generator_randn"])
def test_unreadable_fallback_is_reported(name, tmp_path):
    _ensure_built()
    code = textwrap.dedent(f"""
        import ctypes, sys
        lib = ctypes.CDLL(sys.argv[1], mode=ctypes.RTLD_LOCAL)
        lib.imagine_last_error.restype = ctypes.c_char_p
        rc = lib.{name}(None, 0, 0, None)
        print(rc, lib.imagine_last_error().decode())
    """)
    env = dict(os.environ, IMAGINE_KITCHEN_FALLBACK_LIBRARY=str(tmp_path / "absent.so"))
    r = subprocess.run([sys.executable, "-c", code, SHIM], capture_output=True, text=True,
                       env=env, timeout=120)
    assert r.returncode == 0, r.stderr
    rc, msg = r.stdout.strip().split(" ", 1)
    assert rc == "-1" and "cannot open IMAGINE_KITCHEN_FALLBACK_LIBRARY" in msg
