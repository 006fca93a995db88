"""Stand-ins for the reference suite's helper modules that its component
files import but that the reference does not ship.  Used only by
``tests/golden/make_golden.py`` to run the reference in the build container."""
