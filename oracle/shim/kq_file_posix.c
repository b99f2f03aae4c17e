/*
 * POSIX stand-in for the reference's Win32 read-only file layer
 * (include/kq_file.h, src/kq_file_win32.c:36,150 of Kestrel-Q).
 * Only needed so the reference's GGUF/model translation units link into the
 * oracle library; the oracle never opens a file (synthetic inputs only).
 * Test infrastructure only.
 */
#define _POSIX_C_SOURCE 200809L
#include <fcntl.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>
#include <wchar.h>

#include "kq_file.h"

struct kq_file {
    int descriptor;
    uint64_t size;
};

struct kq_file_view {
    void *mapping;
    size_t mapping_length;
    const unsigned char *data;
    uint64_t offset;
    uint64_t length;
};

static kq_status kq_posix_fail(kq_diagnostic *diagnostic, kq_status status,
                               const char *message) {
    if (diagnostic != NULL) {
        diagnostic->status = status;
        strncpy(diagnostic->message, message, KQ_DIAGNOSTIC_CAPACITY - 1U);
        diagnostic->message[KQ_DIAGNOSTIC_CAPACITY - 1U] = '\0';
    }
    return status;
}

kq_status kq_file_open_readonly(const wchar_t *path, kq_file **out_file,
                                kq_diagnostic *diagnostic) {
    char narrow[4096];
    size_t converted;
    struct stat info;
    kq_file *file;
    int descriptor;
    if (path == NULL || out_file == NULL) {
        return kq_posix_fail(diagnostic, KQ_STATUS_INVALID_ARGUMENT,
                             "path and output are required");
    }
    *out_file = NULL;
    converted = wcstombs(narrow, path, sizeof(narrow) - 1U);
    if (converted == (size_t)-1) {
        return kq_posix_fail(diagnostic, KQ_STATUS_FILE_OPEN_FAILED,
                             "path is not representable");
    }
    narrow[converted] = '\0';
    descriptor = open(narrow, O_RDONLY);
    if (descriptor < 0) {
        return kq_posix_fail(diagnostic, KQ_STATUS_FILE_OPEN_FAILED,
                             "could not open file");
    }
    if (fstat(descriptor, &info) != 0) {
        close(descriptor);
        return kq_posix_fail(diagnostic, KQ_STATUS_FILE_SIZE_FAILED,
                             "could not stat file");
    }
    file = (kq_file *)calloc(1U, sizeof(*file));
    if (file == NULL) {
        close(descriptor);
        return kq_posix_fail(diagnostic, KQ_STATUS_OUT_OF_MEMORY,
                             "out of memory");
    }
    file->descriptor = descriptor;
    file->size = (uint64_t)info.st_size;
    *out_file = file;
    return KQ_STATUS_OK;
}

uint64_t kq_file_size(const kq_file *file) {
    return file == NULL ? 0U : file->size;
}

void kq_file_close(kq_file *file) {
    if (file == NULL) {
        return;
    }
    close(file->descriptor);
    free(file);
}

kq_status kq_file_view_open(kq_file *file, uint64_t offset, uint64_t length,
                            kq_file_view **out_view,
                            kq_diagnostic *diagnostic) {
    long page = sysconf(_SC_PAGESIZE);
    uint64_t aligned;
    uint64_t delta;
    void *mapping;
    kq_file_view *view;
    if (file == NULL || out_view == NULL || length == 0U ||
        offset > file->size || length > file->size - offset || page <= 0) {
        return kq_posix_fail(diagnostic, KQ_STATUS_SPAN_OUT_OF_RANGE,
                             "file view is outside the file");
    }
    *out_view = NULL;
    aligned = offset - (offset % (uint64_t)page);
    delta = offset - aligned;
    mapping = mmap(NULL, (size_t)(length + delta), PROT_READ, MAP_PRIVATE,
                   file->descriptor, (off_t)aligned);
    if (mapping == MAP_FAILED) {
        return kq_posix_fail(diagnostic, KQ_STATUS_FILE_MAP_FAILED,
                             "could not map file view");
    }
    view = (kq_file_view *)calloc(1U, sizeof(*view));
    if (view == NULL) {
        munmap(mapping, (size_t)(length + delta));
        return kq_posix_fail(diagnostic, KQ_STATUS_OUT_OF_MEMORY,
                             "out of memory");
    }
    view->mapping = mapping;
    view->mapping_length = (size_t)(length + delta);
    view->data = (const unsigned char *)mapping + delta;
    view->offset = offset;
    view->length = length;
    *out_view = view;
    return KQ_STATUS_OK;
}

const unsigned char *kq_file_view_data(const kq_file_view *view) {
    return view == NULL ? NULL : view->data;
}

uint64_t kq_file_view_offset(const kq_file_view *view) {
    return view == NULL ? 0U : view->offset;
}

uint64_t kq_file_view_length(const kq_file_view *view) {
    return view == NULL ? 0U : view->length;
}

void kq_file_view_close(kq_file_view *view) {
    if (view == NULL) {
        return;
    }
    munmap(view->mapping, view->mapping_length);
    free(view);
}
