/* Typedef-only stand-in for <GLES2/gl2.h>.  The reference's host-side loader
   (model.cpp, common.cpp, switches.cpp, xformat.cpp) names GL handle types in
   its structs but calls no GL function, so these typedefs are all it needs to
   compile for the oracle's reference build.  No GL library is linked. */
#ifndef VC4B200_GLES2_STUB_H
#define VC4B200_GLES2_STUB_H
typedef unsigned int GLuint;
typedef int GLint;
typedef unsigned int GLenum;
typedef int GLsizei;
typedef float GLfloat;
typedef unsigned char GLubyte;
typedef unsigned char GLboolean;
#endif
