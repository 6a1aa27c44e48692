/* Empty stand-in for <EGL/eglext.h> (see egl.h beside it). */
