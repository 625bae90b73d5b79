"""Drop-in for the reference package of the same name (see the modules inside)."""
