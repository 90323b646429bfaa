"""The reference's unchanged PS firmware driving the B200 engine: its
src/software/main.c, generation.c (the qgen_run loop, generation.c:5-39),
tokenizer.c and utf8_stream.c, compiled from the reference tree by
oracle/Makefile (target ps-loop) with the firmware's own host-simulation
switch and BSP shim headers, and linked with libqwen_b200 through the
platform layer tests/ps_host/b200_board.c (CSR window and embedding copies ->
qwen_b200_csr_write / csr_read / embedding). The firmware loads the real
tokenizer table, runs its 40-token tokenizer self-test (main.c:171-178),
encodes a chat prompt and generates through the CSR protocol; its @TOKEN
transcript must equal greedy generation by the oracle (KV8 + exact mode) on
the same prompt ids."""
import os
import re
import shutil
import subprocess
from pathlib import Path

import pytest

from oracle import ref

pytestmark = pytest.mark.gpu
REPO = Path(__file__).resolve().parents[1]
BIN = REPO / 'oracle' / '_ref' / 'qwen_ps_b200'
TOKEN = REPO / 'oracle' / '_ref' / 'sd' / 'QWEN25' / 'TOKEN.BIN'


def test_unchanged_firmware_transcript_matches_the_oracle(sd_root, tmp_path):
    assert BIN.exists() and TOKEN.exists(), 'the firmware is built by `make -C oracle ps-loop` (needs the reference tree)'
    sd = tmp_path / 'sd'
    (sd / 'QWEN25').mkdir(parents=True)
    for f in (Path(sd_root) / 'QWEN25').iterdir():
        (sd / 'QWEN25' / f.name).symlink_to(f)
    shutil.copy(TOKEN, sd / 'QWEN25' / 'TOKEN.BIN')
    max_new = 4
    session = f'/selftest\n/encode hello B200\n/mode events\n/max {max_new}\nhello B200\n'
    env = dict(os.environ, SIM_SD=str(sd))
    p = subprocess.run([str(BIN)], input=session.encode(), capture_output=True, env=env, timeout=600)
    out = p.stdout.decode('utf-8', 'replace')
    assert p.returncode == 0, out[-2000:] + p.stderr.decode('utf-8', 'replace')[-2000:]
    # the start-up self-test and the /selftest command
    assert out.count('TOKENIZER_SELFTEST_OK 40 tokens') == 2, out[:2000]
    m = re.search(r'@PROMPT (\d+)((?: \d+)+)', out)
    assert m, out
    prompt = [int(t) for t in m.group(2).split()]
    assert len(prompt) == int(m.group(1))
    assert re.search(rf'@BEGIN 1 prompt_tokens={len(prompt)} max_new={max_new}', out), out
    tokens = [int(t) for t in re.findall(r'@TOKEN 1 \d+ (\d+) ', out)]
    end = re.search(r'@END 1 produced=(\d+) reason=(\w+) status=(-?\d+)', out)
    assert end and end.group(3) == '0' and int(end.group(1)) == len(tokens) >= 1, out[-1500:]
    # greedy generation by the oracle on the same ids
    m2 = ref.RefModel(sd_root, capacity=256, mode=ref.KV8 | ref.EXACT)
    try:
        expect, pos, ids = [], 0, prompt
        for _ in range(len(tokens)):
            t = m2.forward(ids, pos)
            expect.append(t)
            pos += len(ids)
            ids = [t]
    finally:
        m2.close()
    assert tokens == expect
