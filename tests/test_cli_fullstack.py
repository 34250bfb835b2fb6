"""CLI commands against real files: checkpoint, dataset, bench, serve, export, generate."""

from pathlib import Path

from underhfs.cli import main
from underhfs.serialization import load_checkpoint, load_manifest


def test_cli_commands(tmp_path=None):
    root = Path(".underhfs-test") if tmp_path is None else Path(tmp_path)
    root.mkdir(exist_ok=True)
    ckpt, binary, data, manifest = (root / n for n in ("tiny.uhfs.json", "tiny.uhfsbin", "sample.txt",
                                                        "tiny.export.json"))
    assert main(["checkpoint", "save-smoke", str(ckpt)]) == 0
    doc = load_checkpoint(ckpt)
    assert doc["metadata"]["model"] == "TransformerLM" and doc["state"]
    assert main(["checkpoint", "inspect", str(ckpt)]) == 0
    assert main(["checkpoint", "save-binary-smoke", str(binary)]) == 0
    assert main(["checkpoint", "inspect-binary", str(binary)]) == 0
    assert main(["dataset", str(data), "--sample"]) == 0 and data.exists()
    assert main(["bench", "--size", "2", "--iterations", "1", "--warmup", "0", "--no-cuda"]) == 0
    assert main(["serve", "--smoke", "--prompt", "hi"]) == 0
    assert main(["serve", "--http-smoke"]) == 0
    assert main(["generate", "--prompt", "hi", "--max-new-tokens", "2"]) == 0
    assert main(["export", str(manifest)]) == 0
    exported = load_manifest(manifest)
    assert exported["model"] == "TransformerLM" and exported["parameters"]
    assert main(["init", str(root / "proj")]) == 0
    if tmp_path is None:
        import shutil

        shutil.rmtree(root)
