"""Extract the sampler golden vectors from the reference's fixtures.

The reference records its sampler tests' tensors as SHA-256 digests of their
contiguous little-endian payload bytes (inference/tests/support/binding.rs:189-200)
in inference/fixtures/qwen-image21-sampling.json (FLUX schedules, flow
algebra, seeded noise, Euler solver runs) and qwen-image21-er-sde.json
(ER-SDE runs: stages 0-4, noise scales, an interior zero sigma), both produced
by the original ComfyUI sampler (comfy/samplers.py, comfy/model_sampling.py).
The harness that drives them is inference/tests/support/qwen_sampling.rs.
This script keeps only what the tests here need (case parameters and
digests) in tests/golden/sampler_fixture.json.  It reads the reference tree and
runs only in the development container; the JSON it writes is committed.

    python tests/golden/make_sampler_golden.py <reference root>
"""
import json
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))


def digest(t):
    return None if t is None else {"sha256": t["payload_sha256"], "shape": t["shape"],
                                   "dtype": t["dtype"]}


def main(root):
    fx = os.path.join(root, "inference", "fixtures")
    sampling = json.load(open(os.path.join(fx, "qwen-image21-sampling.json")))
    er = json.load(open(os.path.join(fx, "qwen-image21-er-sde.json")))
    out = {
        "source": "inference/fixtures/qwen-image21-sampling.json, qwen-image21-er-sde.json",
        "schedules": [{"shift": g["shift"], "sigmas": digest(g["sigmas"]),
                       "cases": [{"method": c["method"], "steps": c["steps"],
                                  "output": digest(c["output"])} for c in g["cases"]]}
                      for g in sampling["schedules"]],
        "algebra": [{"device": c["device"], "dtype": c["dtype"], "scale": c["scale"],
                     **{k: digest(c[k]) for k in ("denoised", "noise", "inverse", "cfg")}}
                    for c in sampling["algebra"]],
        "noises": [{"dtype": c["dtype"], "seed": c["seed"], "output": digest(c["output"])}
                   for c in sampling["noises"]],
        "euler": [{"device": c["device"], "dtype": c["dtype"], "churn": c["churn"],
                   "output": digest(c["output"]),
                   "denoised": [digest(b["denoised"]) for b in c["callbacks"]]}
                  for c in sampling["solvers"]],
        "er_sde": [{"device": c["device"], "dtype": c["dtype"], "max_stage": c["max_stage"],
                    "steps": c["steps"], "noise": c["noise"], "first": c["first"],
                    "float_output": c["float_output"], "explicit_sigmas": c["explicit_sigmas"],
                    "error": ({"class_name": c["error"]["class_name"],
                               "message": c["error"]["message"]}
                              if isinstance(c.get("error"), dict) else None),
                    "output": digest(c.get("output")) if isinstance(c.get("output"), dict) else None,
                    "noises": [digest(n["output"]) for n in c["noises"]],
                    "denoised": [digest(b["denoised"]) for b in c["callbacks"]]}
                   for c in er["cases"]],
        "first_call_x": digest(er["cases"][0]["calls"][0]["x"]),
    }
    with open(os.path.join(HERE, "sampler_fixture.json"), "w") as f:
        json.dump(out, f, indent=0, sort_keys=True)


if __name__ == "__main__":
    if len(sys.argv) != 2:
        raise SystemExit("usage: python tests/golden/make_sampler_golden.py <reference root>")
    main(sys.argv[1])
