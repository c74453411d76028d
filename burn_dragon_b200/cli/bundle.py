"""``python -m burn_dragon_b200.cli.bundle SPEC.toml [--no-resume] [--stop-after NAME]``:
run a multi-stage training bundle (``train.bundle``)."""

from __future__ import annotations

import argparse
import json

from ..train.bundle import BundleOptions, execute_bundle, load_bundle_spec, train_stage


def main(argv=None) -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("spec")
    ap.add_argument("--no-resume", action="store_true")
    ap.add_argument("--stop-after", default=None)
    a = ap.parse_args(argv)
    name, root, stages = load_bundle_spec(a.spec)
    st = execute_bundle(name, root, stages, BundleOptions(not a.no_resume, a.stop_after), train_stage)
    print(json.dumps({"bundle": st["bundle_name"], "latest_completed_stage": st["latest_completed_stage"],
                      "stages": [s["stage_name"] + ":" + s["status"] for s in st["stages"]]}))


if __name__ == "__main__":
    main()
