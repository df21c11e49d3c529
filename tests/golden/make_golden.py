"""Regenerates the golden fixtures in this folder (run in a checkout that has the
Prana reference tree; the fixtures themselves are committed and the tests read
only them).

kquant_encode.npz: seeded f32 blocks and the Q4_K / Q6_K super-blocks the
reference's own encoders produce for them (scripts/convert-to-gguf.py:29-89,
`q4k_encode_block` and `q6k_encode_block`, imported and run unchanged).  They
pin this repository's synthetic-model encoders byte for byte.

Usage: python tests/golden/make_golden.py path/to/reference/checkout
"""
import importlib.util
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent


def load_reference_encoders(root: Path):
    spec = importlib.util.spec_from_file_location("prana_convert_to_gguf", root / "scripts" / "convert-to-gguf.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)  # the script's main() only runs under __main__
    return mod


def blocks(rng: np.random.Generator) -> np.ndarray:
    """Seeded 256-value blocks: model-like normals at several scales plus edge shapes."""
    out = [rng.normal(0.0, s, 256) for s in (0.02, 0.02, 0.02, 0.1, 1.0, 5.0) for _ in range(4)]
    out += [np.zeros(256), np.full(256, 0.5), np.full(256, -0.25), -np.abs(rng.normal(0, 0.02, 256)),
            np.abs(rng.normal(0, 0.02, 256)), rng.uniform(-1, 1, 256) * 1e-6, rng.standard_t(2, 256) * 0.05]
    one_hot = np.zeros(256)
    one_hot[37] = 3.0
    out.append(one_hot)
    return np.stack(out).astype(np.float32)


def main(root: str) -> None:
    ref = load_reference_encoders(Path(root))
    x = blocks(np.random.default_rng(20240611))
    q4k = np.stack([np.frombuffer(ref.q4k_encode_block([float(v) for v in b]), np.uint8) for b in x])
    q6k = np.stack([np.frombuffer(ref.q6k_encode_block([float(v) for v in b]), np.uint8) for b in x])
    assert q4k.shape[1] == 144 and q6k.shape[1] == 210
    np.savez_compressed(HERE / "kquant_encode.npz", x=x, q4_k=q4k, q6_k=q6k)
    print(f"wrote {len(x)} blocks to {HERE / 'kquant_encode.npz'}")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit(__doc__)
    main(sys.argv[1])
