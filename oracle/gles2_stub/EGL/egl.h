/* Typedef-only stand-in for <EGL/egl.h>.  The reference's class GPU
   (engine/src/gpu.h) keeps EGL handles as members; the oracle's build of the
   reference layer loop (oracle/ref_session.cpp) constructs that class without
   ever calling EGL, so the handle types and their null values are all it
   needs.  No EGL library is linked. */
#ifndef VC4B200_EGL_STUB_H
#define VC4B200_EGL_STUB_H
typedef void* EGLDisplay;
typedef void* EGLContext;
typedef void* EGLSurface;
typedef void* EGLConfig;
typedef void* EGLImageKHR;
typedef int EGLint;
typedef unsigned int EGLBoolean;
typedef unsigned int EGLenum;
#define EGL_NO_DISPLAY ((EGLDisplay)0)
#define EGL_NO_CONTEXT ((EGLContext)0)
#define EGL_NO_SURFACE ((EGLSurface)0)
#define EGL_NO_IMAGE_KHR ((EGLImageKHR)0)
#endif
