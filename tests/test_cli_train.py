from underhfs.cli import main


def test_train_smoke_cli():
    assert main(["train", "--smoke", "--steps", "1"]) == 0


def test_train_without_mode_returns_2():
    assert main(["train"]) == 2
