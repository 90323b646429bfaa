"""Test helper: the reference's generation loop, src/software/generation.c:5-39,
restated in Python so tests can drive any CSR backend (the B200 engine through
the C ABI, or a fake) exactly as the unchanged PS firmware would."""
CAPACITY, VOCAB = 256, 151936


class Result:
    def __init__(self):
        self.produced, self.eos, self.last_status = 0, 0, 0


def qgen_run(ops, prompt, max_new, ticks_per_second=1_000_000):
    """Returns (status, Result, tokens). Status codes of generation.h:16."""
    res, tokens = Result(), []
    count = len(prompt)
    if not count or not max_new or max_new >= CAPACITY or count > CAPACITY - max_new:
        return -1, res, tokens
    if any(t >= VOCAB for t in prompt):
        return -1, res, tokens
    for row, tok in enumerate(prompt):
        ops.embedding(tok, row)
    position, rows = 0, count
    for iteration in range(max_new):
        ops.write(0x80, int(iteration != 0))
        ops.write(0x88, rows)
        ops.write(0x90, position + rows)
        ops.write(0x98, position)
        start = ops.ticks()
        ops.write(0x10, 1)
        while True:
            res.last_status = ops.read(0x18)
            now = ops.ticks()
            if res.last_status & (1 << 3):
                return -3, res, tokens
            if (res.last_status & 0x46) == 0x44:
                break
            if now - start > 1800 * ticks_per_second:
                return -2, res, tokens
            ops.wait()
        value = ops.read(0x1f8)
        if value >= VOCAB:
            return -4, res, tokens
        if ops.token(iteration, value, now - start):
            return -5, res, tokens
        tokens.append(value)
        res.produced += 1
        if value in (151643, 151645):
            res.eos = 1
            break
        position += rows
        rows = 1
        if iteration + 1 < max_new:
            ops.embedding(value, 0)
    return 0, res, tokens


class EngineOps:
    """qgen_ops bound to a libqwen_b200 handle (write/read/embedding from the C ABI)."""

    def __init__(self, lib, handle):
        import time
        self.lib, self.h, self._time = lib, handle, time

    def write(self, off, value):
        self.lib.qwen_b200_csr_write(self.h, off, value)

    def read(self, off):
        return self.lib.qwen_b200_csr_read(self.h, off)

    def embedding(self, token, row):
        self.lib.qwen_b200_embedding(self.h, token, row)

    def ticks(self):
        return int(self._time.monotonic() * 1_000_000)

    def wait(self):
        self._time.sleep(0.0001)  # main.c:54 usleep(100)

    def token(self, iteration, token, elapsed):
        return 0
