"""The generation-loop contract above the boundary (src/software/generation.c:5-39)
against a scripted fake PL, including the reference harness's fault injection
(src/software/tests/board_sim.c:40-147: timeout, pl_error, invalid_token) — the
loop the engine's CSR emulation must satisfy, checked without a GPU."""
import pytest

from qgen import qgen_run


class FakePL:
    """Scripted tokens; START latches a result, 0x18 is busy twice then done."""

    def __init__(self, tokens, fault=None):
        self.tokens, self.fault = tokens, fault
        self.regs, self.ids, self.iteration, self.polls, self.t = {}, {}, -1, 0, 0
        self.starts = []

    def write(self, off, v):
        self.regs[off] = v
        if off == 0x10 and v == 1:
            self.iteration = 0 if self.regs[0x80] == 0 else self.iteration + 1
            self.polls = 0
            self.starts.append((self.regs[0x80], self.regs[0x88], self.regs[0x90], self.regs[0x98]))

    def read(self, off):
        if off == 0x18:
            if self.fault == 'timeout':
                self.t += 600_000_000
                return 2
            if self.fault == 'pl_error':
                return 8
            self.polls += 1
            return 2 if self.polls < 3 else 0x44
        if off == 0x1f8:
            return 151936 if self.fault == 'invalid_token' else self.tokens[min(self.iteration, len(self.tokens) - 1)]
        return self.regs.get(off, 0)

    def embedding(self, token, row):
        self.ids[row] = token

    def ticks(self):
        self.t += 100
        return self.t

    def wait(self):
        self.t += 100

    def token(self, iteration, token, elapsed):
        return 0


def test_prefill_then_decode_register_sequence():
    pl = FakePL([11, 12, 13])
    status, res, toks = qgen_run(pl, [5, 6, 7, 8], 3)
    assert status == 0 and toks == [11, 12, 13] and res.produced == 3 and not res.eos
    # prefill of 4 rows at position 0, then 1-row decodes (generation.c:13-16,34-35)
    assert pl.starts == [(0, 4, 4, 0), (1, 1, 5, 4), (1, 1, 6, 5)]
    assert pl.ids[0] == 12  # last fed token (embedding row 0)


def test_eos_stops_generation():
    status, res, toks = qgen_run(FakePL([3, 151645, 4]), [1], 5)
    assert status == 0 and res.eos == 1 and toks == [3, 151645]


@pytest.mark.parametrize('fault,code', [('timeout', -2), ('pl_error', -3), ('invalid_token', -4)])
def test_fault_injection(fault, code):
    status, res, toks = qgen_run(FakePL([1], fault), [1, 2], 2)
    assert status == code and not toks


@pytest.mark.parametrize('prompt,max_new', [([], 4), ([1], 0), ([1], 256), ([1] * 250, 10), ([151936], 1)])
def test_bad_requests(prompt, max_new):
    assert qgen_run(FakePL([1]), prompt, max_new)[0] == -1
