"""Examples and the standalone server launcher: the example scripts parse,
and the launcher routes its subcommands (and bare flags, meaning serve) to
the CLI."""

import ast
import os

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
EXAMPLES = ["basic_inference.py", "batch_processing.py", "multi_gpu.py", "openai_server.py",
            "streaming.py"]


@pytest.mark.parametrize("name", EXAMPLES)
def test_example_parses(name):
    src = open(os.path.join(ROOT, "examples", name)).read()
    tree = ast.parse(src)
    assert any(isinstance(n, ast.FunctionDef) and n.name == "main" for n in tree.body)


def test_server_launcher_routes_to_cli(monkeypatch):
    import swiftllm_b200.cli as cli
    from swiftllm_b200.server import __main__ as launcher
    seen = []
    monkeypatch.setattr(cli, "main", lambda argv=None: seen.append(list(argv)) or 0)
    assert launcher.main(["--model", "tiny-llama", "--port", "9"]) == 0
    assert launcher.main(["info", "--model", "tiny-llama"]) == 0
    assert seen == [["serve", "--model", "tiny-llama", "--port", "9"], ["info", "--model", "tiny-llama"]]
