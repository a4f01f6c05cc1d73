"""The riding caller's step order on the CPU (include/imi_flow_cuda.h against a fake of the C-ABI calls it makes,
tests/flow_fake.cpp): flow.cpp:114-126 rides every text word on a voice frame's step while both have work, then
steps the one left alone; a text part ends at its cap or at the stop word, and the end callback may start the next
part (flow.cpp:57-76)."""
import os
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def fake(tmp_path_factory):
    exe = str(tmp_path_factory.mktemp("flow") / "flow_fake")
    r = subprocess.run(["g++", "-std=c++17", "-O1", "-Wall", "-Wextra", "-Werror", "-I", os.path.join(ROOT, "include"),
                        os.path.join(ROOT, "tests", "flow_fake.cpp"), "-o", exe], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr

    def run(ride, frames, cap1, cap2, stop_at=-1):
        out = subprocess.run([exe, str(int(ride)), str(frames), str(cap1), str(cap2), str(stop_at)],
                             capture_output=True, text=True, check=True).stdout.splitlines()
        picks = [int(x) for x in out[-2].split()[1:]]
        counts = tuple(int(x) for x in out[-1].split()[1:])
        return out[:-2], picks, counts
    return run


def test_every_word_rides_while_the_voice_speaks(fake):
    log, picks, counts = fake(True, 5, 3, 2)
    assert picks == [110, 111, 112, 120, 121]          # part 1 from the prompt at 10, part 2 from the re-prompt at 20
    assert counts == (5, 0, 0)
    steps = [line for line in log if line.startswith("step")]
    assert steps == ["step2 voice -1 hidden + text %d logits" % w for w in (110, 111, 112, 120, 121)]
    assert log.index("end of part 1") < log.index("step2 voice -1 hidden + text 120 logits")


def test_alone_gives_the_same_words_and_frames(fake):
    log_r, picks_r, _ = fake(True, 7, 3, 2)
    log_a, picks_a, counts_a = fake(False, 7, 3, 2)
    assert picks_a == picks_r and counts_a == (0, 5, 7)
    # alone: each round steps the voice, then the text word (flow.cpp:123-124)
    steps = [line for line in log_a if line.startswith("step")]
    assert steps[:2] == ["step voice -1 hidden", "step text 110 logits"]
    assert steps.count("step voice -1 hidden") == 7


def test_the_one_left_steps_alone(fake):
    _, picks, counts = fake(True, 2, 3, 2)              # speech ends first: the text goes on alone
    assert picks == [110, 111, 112, 120, 121] and counts == (2, 3, 0)
    _, picks, counts = fake(True, 9, 3, 2)              # the text ends first: the voice goes on alone
    assert counts == (5, 0, 4)


def test_stop_word_ends_a_part(fake):
    _, picks, counts = fake(True, 8, 5, 2, stop_at=12)  # the pick at text position 12 is the stop word
    assert picks == [110, 111, 120, 121] and counts == (4, 0, 4)
