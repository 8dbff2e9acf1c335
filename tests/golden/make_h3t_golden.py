"""Record the reference writer's output for two small synthetic stores: run the REFERENCE h3t writer
(h3turbo/h3/writer.py) on the same seeded tensors this package's tests write, and store each file's size and sha256 in
tests/golden/h3t_golden.json.  tests/test_store.py checks that this package's writer produces byte-identical files.

Usage:  python tests/golden/make_h3t_golden.py /path/to/reference
"""
import hashlib
import json
import sys
import tempfile
from pathlib import Path

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent))

CASES = {"fp8_g16": ("fp8", 16), "fp16_g128": ("fp16", 128)}


def config(group):
    from minimax_h3_turbo_b200.h3.config import H3Config

    return H3Config(hidden=256, layers=3, refiner_layers=0, heads=2, head_dim=128, ffn=512, text_dim=64, video_channels=4,
                    audio_channels=8, quant_group=group)


def main(ref_root: str) -> None:
    import conftest  # noqa: F401  -- registers this package (the synthetic tensors)
    from minimax_h3_turbo_b200.h3.synth import synthetic_store_tensors

    sys.path.insert(0, ref_root)
    from h3turbo.h3 import config as ref_config  # noqa: E402  (the reference)
    from h3turbo.h3 import writer as ref_writer  # noqa: E402

    out = {}
    with tempfile.TemporaryDirectory() as d:
        for name, (fmt, group) in CASES.items():
            cfg = config(group)
            tensors = {k: (v.read() if hasattr(v, "read") else v)
                       for k, v in synthetic_store_tensors(cfg, group=group, scale_dtype=fmt, seed=3).items()}
            path = Path(d) / f"{name}.h3t"
            ref_writer.write_h3t(path, ref_config.H3Config.from_json(cfg.to_json()), tensors)
            raw = path.read_bytes()
            out[name] = {"format": fmt, "group": group, "seed": 3, "size": len(raw), "sha256": hashlib.sha256(raw).hexdigest()}
    (HERE / "h3t_golden.json").write_text(json.dumps(out, indent=1) + "\n")
    print(out)


if __name__ == "__main__":
    main(sys.argv[1])
