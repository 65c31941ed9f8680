#!/usr/bin/env python3
"""Install the reference implementation into baseline/_ref (git-ignored) for `bench.py --impl reference`.

1. The prescribed offline pip install (`pip install --no-index --no-build-isolation --find-links /opt/wheelhouse
   --target baseline/_ref SRC`). The reference is a research repository without package metadata, so pip stops with
   "not installable".
2. Then the reference's importable package, `code/kva` (plain PyTorch; imports torch and safetensors only), is
   copied file for file, unmodified, to baseline/_ref/kva, and baseline/_ref/INSTALL.json records the pip outcome and
   every copied file's sha256 (the reference arm re-hashes them before it runs and refuses a modified copy). Its
   protocol file and paper run configs are copied beside it as data for the configuration-compatibility tests.

    python baseline/install_reference.py SRC        # SRC: the reference checkout (its root, holding code/kva)
"""
import hashlib
import json
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
DST = HERE / "_ref"


def sha256(p):
    return hashlib.sha256(Path(p).read_bytes()).hexdigest()


def main(argv):
    if len(argv) != 1:
        sys.exit(__doc__)
    src = Path(argv[0]).resolve()
    DST.mkdir(parents=True, exist_ok=True)
    pip = subprocess.run([sys.executable, "-m", "pip", "install", "--no-index", "--no-build-isolation",
                          "--find-links", "/opt/wheelhouse", "--target", str(DST), str(src)],
                         capture_output=True, text=True)
    tail = (pip.stderr or pip.stdout).strip().splitlines()[-3:]
    record = dict(pip_returncode=pip.returncode, pip_tail=tail, source="code/kva", files={})
    pkg = src / "code" / "kva"
    if pip.returncode != 0:
        if not (pkg / "__init__.py").is_file():
            sys.exit(f"pip failed and {pkg} holds no package: {tail}")
        target = DST / "kva"
        if target.exists():
            shutil.rmtree(target)
        for f in sorted(pkg.rglob("*.py")):
            rel = f.relative_to(pkg)
            (target / rel).parent.mkdir(parents=True, exist_ok=True)
            shutil.copyfile(f, target / rel)
            record["files"][rel.as_posix()] = sha256(f)
        for extra in ("LICENSE", "protocol.json"):
            if (src / "code" / extra).is_file():
                shutil.copyfile(src / "code" / extra, DST / extra)
                record["files_data"] = dict(record.get("files_data", {}), **{extra: sha256(src / "code" / extra)})
        fin = src / "code" / "finals"               # the battery's cells and their schema: compatibility test data
        if fin.is_dir():
            dst_fin = DST / "finals"
            if dst_fin.exists():
                shutil.rmtree(dst_fin)
            (dst_fin / "cells").mkdir(parents=True)
            for f in sorted((fin / "cells").glob("*.json")) + [fin / "cell.schema.json"]:
                if f.is_file():
                    to = dst_fin / ("cells" if f.parent.name == "cells" else "") / f.name
                    shutil.copyfile(f, to)
                    record.setdefault("files_data", {})["finals/" + to.relative_to(dst_fin).as_posix()] = sha256(f)
            for extra in ("stats.py",):              # its statistics, run as an oracle by the tests
                if (fin / extra).is_file():
                    shutil.copyfile(fin / extra, dst_fin / extra)
                    record["files"]["../finals/" + extra] = sha256(fin / extra)
            (dst_fin / "lib").mkdir()                # its cell-to-config code, run as an oracle by the tests
            for f in sorted((fin / "lib").glob("*.py")):
                shutil.copyfile(f, dst_fin / "lib" / f.name)
                record["files"]["../finals/lib/" + f.name] = sha256(f)
        cfg_src = src / "code" / "configs"           # the paper's run configs: compatibility test data
        if cfg_src.is_dir():
            if (DST / "configs").exists():
                shutil.rmtree(DST / "configs")
            shutil.copytree(cfg_src, DST / "configs")
            for f in sorted((DST / "configs").rglob("*.json")):
                record.setdefault("files_data", {})["configs/" + f.relative_to(DST / "configs").as_posix()] = sha256(f)
    (DST / "INSTALL.json").write_text(json.dumps(record, indent=1))
    print(json.dumps(dict(pip_returncode=pip.returncode, pip=tail[-1] if tail else "", copied=len(record["files"]))))


if __name__ == "__main__":
    main(sys.argv[1:])
