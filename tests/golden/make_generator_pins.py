"""Writes tests/golden/generator.json: the first draws of the seeded input
generator (oracle/oracle.cpp, SplitMix64-seeded xoshiro256** and Box-Muller),
so that tests notice if the generator ever changes.

    python tests/golden/make_generator_pins.py
"""
import json
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "..", "..", "oracle"))
import oracle as orc  # noqa: E402


def main():
    r = orc.Rng(0)
    first = [int(orc.lib().orc_rng_next(r.state.ctypes.data_as(orc._u64p))) for _ in range(2)]
    n = orc.Rng(1).normal(4)
    json.dump({"xoshiro256ss_seed0_first2": first,
               "normal_seed1_first4": [float(x) for x in n]},
              open(os.path.join(HERE, "generator.json"), "w"), indent=1)


if __name__ == "__main__":
    main()
