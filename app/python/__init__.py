"""Drop-in names for the reference's `app.python` modules, served by directaccesskernel_b200."""
