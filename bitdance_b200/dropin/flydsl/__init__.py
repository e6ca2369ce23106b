"""Stand-in for the FlyDSL package the reference's scripts import (flydsl 0.1.9 for gfx950 in
the reference's environment, REPRODUCE.md:70-72). Only the names those scripts use exist."""
