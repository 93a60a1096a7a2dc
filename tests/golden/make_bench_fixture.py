"""Generate tests/golden/bench_decode_ids.json: the first greedy ids the CPU
oracle decodes after each bench config's prompt, on the bench's own seeded
synthetic model (written here with the same generator and seed, on the CPU).

bench.py compares its decode head with these ids and fails when they differ.
The file also records each model file's sha256, so a mismatch between the
bench's model bytes and the fixture's is reported as such rather than as a
parity failure.  Run: python tests/golden/make_bench_fixture.py [config ...]
(about 10 minutes on 8 cores for the three configs below)."""
import hashlib
import json
import os
import sys
import time

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

import numpy as np  # noqa: E402

# config -> (synth spec, prompt tokens, max context): bench.py CONFIGS / MAX_CONTEXT
CASES = {
    "qwen3-0.6b-q4_k_m": ("qwen3-0.6b", 512, 2048),
    "smollm2-135m-q4_k_m": ("smollm2-135m", 32, 512),
    "qwen3-0.6b-q8_0": ("qwen3-0.6b-q8", 1920, 2048),
}
N_IDS = 8


def sha256(path):
    h = hashlib.sha256()
    with open(path, "rb") as f:
        for chunk in iter(lambda: f.read(1 << 24), b""):
            h.update(chunk)
    return h.hexdigest()


def main(names):
    from chonklm_b200.synth import SPECS, write_synthetic_gguf
    from oracle import oracle
    out_path = os.path.join(HERE, "bench_decode_ids.json")
    out = json.load(open(out_path)) if os.path.exists(out_path) else {}
    tmp = os.environ.get("CK_FIXTURE_DIR", "/tmp/ck_fixture")
    os.makedirs(tmp, exist_ok=True)
    for name in names:
        spec, plen, ctx = CASES[name]
        path = os.path.join(tmp, f"{spec}.gguf")
        if not os.path.exists(path):
            write_synthetic_gguf(SPECS[spec], path, seed=0, device="cpu")
        prompt = np.random.default_rng(1).integers(0, SPECS[spec].vocab, size=plen).tolist()
        t0 = time.time()
        m = oracle.OracleModel(path, max_context=ctx)
        ids = oracle.generate(m, prompt, N_IDS)
        m.close()
        out[name] = {"spec": spec, "prompt_seed": 1, "prompt_len": plen, "ids": [int(i) for i in ids],
                     "gguf_sha256": sha256(path)}
        print(name, out[name]["ids"], f"{time.time() - t0:.0f}s", flush=True)
        with open(out_path, "w") as f:
            json.dump(out, f, indent=1, sort_keys=True)


if __name__ == "__main__":
    main(sys.argv[1:] or list(CASES))
