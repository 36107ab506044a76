/*
 * Minimal stand-in for libpng's header, used only when the reference's
 * src/mesh.cpp is compiled into the test oracle (oracle/_ref). libpng is not
 * installed in this image and the synthetic meshes carry no textures, so every
 * entry point below reports failure: png_create_read_struct returns NULL and
 * the reference's loadPngTexture (mesh.cpp:38-50) then returns without a
 * texture. Nothing here decodes PNG data.
 */
#pragma once
#include <csetjmp>
#include <cstddef>
#include <cstdio>

typedef unsigned int png_uint_32;
typedef std::size_t png_size_t;
typedef unsigned char* png_bytep;
typedef struct png_stub_struct { std::jmp_buf jb; }* png_structp;
typedef struct png_stub_info { int unused; }* png_infop;

#define PNG_LIBPNG_VER_STRING "stub"
#define PNG_COLOR_TYPE_GRAY 0
#define PNG_COLOR_TYPE_PALETTE 3
#define PNG_COLOR_TYPE_GRAY_ALPHA 4
#define PNG_COLOR_MASK_ALPHA 4
#define PNG_INFO_tRNS 0x0010
#define png_jmpbuf(p) ((p)->jb)

inline png_structp png_create_read_struct(const char*, void*, void*, void*) { return nullptr; }
inline png_infop png_create_info_struct(png_structp) { return nullptr; }
inline void png_destroy_read_struct(png_structp*, png_infop*, void*) {}
inline void png_init_io(png_structp, std::FILE*) {}
inline void png_read_info(png_structp, png_infop) {}
inline png_uint_32 png_get_IHDR(png_structp, png_infop, png_uint_32*, png_uint_32*, int*, int*,
                                int*, int*, int*) { return 0; }
inline void png_set_strip_16(png_structp) {}
inline void png_set_palette_to_rgb(png_structp) {}
inline void png_set_expand_gray_1_2_4_to_8(png_structp) {}
inline png_uint_32 png_get_valid(png_structp, png_infop, png_uint_32) { return 0; }
inline void png_set_tRNS_to_alpha(png_structp) {}
inline void png_set_gray_to_rgb(png_structp) {}
inline void png_set_strip_alpha(png_structp) {}
inline void png_read_update_info(png_structp, png_infop) {}
inline png_size_t png_get_rowbytes(png_structp, png_infop) { return 0; }
inline void png_read_image(png_structp, png_bytep*) {}
